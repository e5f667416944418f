"""numpy restatement of the GRINQH hot path (CPU oracle; test infrastructure only).

Every function cites the reference file:line it restates (paths relative to the
reference project root). Integer / byte work is bit-exact; the float paths are
computed in float64 from the same fp32-exact operands the reference kernels see,
then rounded to the output dtype, so that they serve as a tolerance oracle for
both the reference's Triton kernels and this build's CUDA kernels.

bf16 values travel as uint16 bit patterns (numpy has no bfloat16); fp16 values
are numpy float16.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_bits_to_f32", "f32_to_bf16_bits", "to_f32", "round_to_dtype",
    "preshuffle", "postshuffle", "shifted_words", "pack_words", "pack_codes",
    "unpack", "unpack_codes", "grade", "zone_bias", "bias_table",
    "masked_codes", "graded_gemv", "union_gemv", "looped_gemv", "graded_rows", "dense_weight", "dense",
    "gemm_or_gemv", "ct_pack_to_int32", "ct_unpack_from_int32",
    "rtn_quantize", "make_activations", "quantile_thresholds",
]


# ----------------------------------------------------------------------------- dtypes
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch's .to(bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Activation / scale storage -> float32 (exact): dtype is 'bf16' or 'f16'."""
    if dtype == "bf16":
        return bf16_bits_to_f32(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float16).astype(np.float32)
    raise ValueError(dtype)


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """float -> storage of ``dtype`` (uint16 bits for bf16, float16 for f16), RNE."""
    x32 = np.asarray(x, dtype=np.float64).astype(np.float32)
    if dtype == "bf16":
        return f32_to_bf16_bits(x32)
    if dtype == "f16":
        return x32.astype(np.float16)
    raise ValueError(dtype)


# ----------------------------------------------------------------------------- layout
def preshuffle(w: np.ndarray) -> np.ndarray:
    """Column permutation (K,16,N/16)->(K,N/16,16). grinqh/utils.py:17-22."""
    k, n = w.shape
    if n % 16:
        raise ValueError("N must be divisible by 16 for this layout.")
    return np.ascontiguousarray(w.reshape(k, 16, n // 16).transpose(0, 2, 1)).reshape(k, n)


def postshuffle(w: np.ndarray) -> np.ndarray:
    """Inverse of :func:`preshuffle`. grinqh/utils.py:25-30."""
    k, n = w.shape
    if n % 16:
        raise ValueError("N must be divisible by 16 for this layout.")
    return np.ascontiguousarray(w.reshape(k, n // 16, 16).transpose(0, 2, 1)).reshape(k, n)


def shifted_words(codes: np.ndarray, max_bits: int) -> np.ndarray:
    """int8 codes (K,N) -> preshuffled, ``<< (8-b)`` shifted uint32 words (K,N/4).

    grinqh/grinqh.py:204-207 (``grinqh_input_preshuffle`` then ``<< shift_amt``
    on int8, which wraps modulo 256)."""
    shift = 8 - max_bits
    sh = preshuffle(np.asarray(codes, dtype=np.int8))
    b = (sh.astype(np.int16) << shift).astype(np.int64) & 0xFF
    return np.ascontiguousarray(b.astype(np.uint8)).view(np.uint32)


def pack_words(a: np.ndarray, max_bits: int) -> np.ndarray:
    """Bit-plane pack, restating ``_pack_kernel_uint32`` (grinqh/utils.py:100-122)
    with the host wrapper ``pack_triton`` (utils.py:125-146).

    ``a``: (K, Nw) uint32 (4 shifted code bytes per word). Returns
    (K, (b/2) * Nw/4) uint32: output word ``zone*N_zone + j`` holds, in byte
    lane L at bits (7-2i, 6-2i), bits (7-2*zone, 6-2*zone) of byte L of input
    word ``4j+i``.
    """
    a = np.asarray(a, dtype=np.uint32)
    k, nw = a.shape
    n_zone = nw // 4
    nz = max_bits // 2
    out = np.zeros((k, nz * n_zone), dtype=np.uint32)
    quad = a[:, : 4 * n_zone].reshape(k, n_zone, 4)
    for z in range(nz):
        src = np.uint32((3 - z) * 2)
        acc = np.zeros((k, n_zone), dtype=np.uint32)
        for i in range(4):
            dst = np.uint32((3 - i) * 2)
            acc |= ((quad[:, :, i] >> src) & np.uint32(0x03030303)) << dst
        out[:, z * n_zone:(z + 1) * n_zone] = acc
    return out


def pack_codes(codes: np.ndarray, max_bits: int) -> np.ndarray:
    """Load-time transform of ``process_weights_after_loading``
    (grinqh/grinqh.py:202-211): preshuffle, shift, pack."""
    return pack_words(shifted_words(codes, max_bits), max_bits)


def unpack(packed: np.ndarray, max_bits: int, original_n: int) -> np.ndarray:
    """``unpack_pyt`` (grinqh/utils.py:149-177) over every row: (K, N) uint8 of the
    preshuffled column order, each byte ``shifted_code >> (8-b)`` (unsigned)."""
    p = np.asarray(packed, dtype=np.uint32)
    k = p.shape[0]
    nz = max_bits // 2
    n_zone = original_n // 4
    planes = p[:, : n_zone * nz].reshape(k, nz, n_zone)
    res = np.zeros((k, n_zone, 4), dtype=np.uint32)
    for z in range(nz):
        merge = np.uint32(2 * (nz - 1 - z))
        for i, s in enumerate((6, 4, 2, 0)):
            res[:, :, i] += ((planes[:, z, :] >> np.uint32(s)) & np.uint32(0x03030303)) << merge
    return np.ascontiguousarray(res.reshape(k, n_zone * 4)).view(np.uint8)


def unpack_codes(packed: np.ndarray, max_bits: int, original_n: int) -> np.ndarray:
    """Signed codes in the original column order, as the dense path recovers them
    (grinqh/kernel.py:571-576: unpack, sign-extend, postshuffle)."""
    shift = 8 - max_bits
    u = unpack(packed, max_bits, original_n).astype(np.int16)
    signed = ((u << shift).astype(np.int64) & 0xFF).astype(np.uint8).view(np.int8).astype(np.int16) >> shift
    return postshuffle(signed.astype(np.int8))


# ----------------------------------------------------------------------------- grading
def grade(x_f32: np.ndarray, thresholds, max_bits: int) -> np.ndarray:
    """Zone mask per activation element: bit z set iff ``fp32|x| > fp32(t_z)`` for
    z < b/2 (strict). grinqh/kernel.py:100-116 (thresholds are fp32 constexprs;
    Triton compares in fp32), tests/test_grinqh_ops.py:37,46."""
    ax = np.abs(np.asarray(x_f32, dtype=np.float32))
    m = np.zeros(ax.shape, dtype=np.uint8)
    for z in range(max_bits // 2):
        m |= (ax > np.float32(thresholds[z])).astype(np.uint8) << z
    return m


def bias_table(max_bits: int) -> np.ndarray:
    """Mid-point bias for each of the 16 zone masks (grinqh/kernel.py:73-82,108-114):
    ``sum over active z of Delta_z``, ``Delta_z = B_z - B_{z-1}``,
    ``B_z = 2^(b-1) >> (2z+2)``, ``B_{-1} = 0``; zones z >= b/2 never count."""
    base = 1 << (max_bits - 1)
    b = [base >> (2 * z + 2) for z in range(4)]
    delta = [b[0], b[1] - b[0], b[2] - b[1], b[3] - b[2]]
    tab = np.zeros(16, dtype=np.int32)
    for mask in range(16):
        tab[mask] = sum(delta[z] for z in range(max_bits // 2) if mask >> z & 1)
    return tab


def zone_bias(mask: np.ndarray, max_bits: int) -> np.ndarray:
    return bias_table(max_bits)[np.asarray(mask, dtype=np.int64)]


def masked_codes(codes: np.ndarray, row_mask: np.ndarray, max_bits: int) -> np.ndarray:
    """Masked weight ``int8(byte & zone_bits) >> (8-b)`` per row k, where the byte is
    the shifted code and zone_bits = OR over active z of ``0xC0 >> 2z``.
    grinqh/kernel.py:120-146 (inactive planes load as 0) and the test oracle
    tests/test_grinqh_ops.py:40-53."""
    shift = 8 - max_bits
    byte = (np.asarray(codes, dtype=np.int16) << shift).astype(np.int64) & 0xFF
    bits = np.zeros(np.asarray(row_mask).shape, dtype=np.int64)
    for z in range(4):
        bits |= ((np.asarray(row_mask, dtype=np.int64) >> z) & 1) * (0xC0 >> (2 * z))
    mb = (byte & bits[:, None]).astype(np.uint8).view(np.int8).astype(np.int32)
    return mb >> shift


def _scales_rows(scales_f32: np.ndarray, k: int, group_size: int) -> np.ndarray:
    return np.repeat(np.asarray(scales_f32, dtype=np.float64), group_size, axis=0)[:k]


def graded_gemv(x_f32: np.ndarray, codes: np.ndarray, scales_f32: np.ndarray,
                thresholds, max_bits: int, group_size: int) -> np.ndarray:
    """M == 1 graded GEMV of ``grinqh_gemv_uint32_packed`` (grinqh/kernel.py:39-167):
    ``y[n] = sum_k s[k//g, n] * x_k * (w_masked[k,n] + bias_k)`` (float64, before
    the fp32->dtype cast of kernel.py:706)."""
    x = np.asarray(x_f32, dtype=np.float32).reshape(-1)
    mask = grade(x, thresholds, max_bits)
    w = masked_codes(codes, mask, max_bits).astype(np.float64) + zone_bias(mask, max_bits)[:, None]
    s = _scales_rows(scales_f32, w.shape[0], group_size)
    return (x.astype(np.float64)[None, :] @ (w * s))[0]


def union_gemv(x_f32: np.ndarray, codes: np.ndarray, scales_f32: np.ndarray,
               thresholds, max_bits: int, group_size: int) -> np.ndarray:
    """Small-batch GEMV graded by the union ``max_m |x[m,k]|``
    (``grinqh_gemv_uint32_packed_batch_union``, grinqh/kernel.py:170-360)."""
    x = np.asarray(x_f32, dtype=np.float32)
    umax = np.abs(x).max(axis=0)
    mask = grade(umax, thresholds, max_bits)
    w = masked_codes(codes, mask, max_bits).astype(np.float64) + zone_bias(mask, max_bits)[:, None]
    s = _scales_rows(scales_f32, w.shape[0], group_size)
    return x.astype(np.float64) @ (w * s)


def looped_gemv(x_f32: np.ndarray, codes, scales_f32, thresholds, max_bits, group_size):
    """Per-token graded rows (each row of x graded by itself): the reference's M==1
    path applied token by token (tests/test_grinqh_ops.py:271)."""
    x = np.asarray(x_f32, dtype=np.float32)
    return np.stack([graded_gemv(x[m], codes, scales_f32, thresholds, max_bits, group_size)
                     for m in range(x.shape[0])])


def graded_rows(x_f32: np.ndarray, codes: np.ndarray, scales_f32: np.ndarray,
                thresholds, max_bits: int, group_size: int, k_chunk: int = 512) -> np.ndarray:
    """Same result as :func:`looped_gemv` (every row of x graded by itself,
    grinqh/kernel.py:100-158 per token), evaluated for many rows at once: the masked
    weight of row k depends only on that row's zone mask, so for each mask value that
    occurs the rows' activations with that mask multiply one masked weight matrix.
    Processed in K chunks of ``k_chunk`` rows (a multiple of ``group_size``) so the
    float64 matrices stay small. Float64 accumulation."""
    x = np.asarray(x_f32, dtype=np.float32).reshape(-1, np.asarray(x_f32).shape[-1])
    m_all = grade(x, thresholds, max_bits)
    k_total, n = codes.shape
    assert k_chunk % group_size == 0
    y = np.zeros((x.shape[0], n), dtype=np.float64)
    bias = bias_table(max_bits)
    for k0 in range(0, k_total, k_chunk):
        k1 = min(k_total, k0 + k_chunk)
        s = _scales_rows(scales_f32[k0 // group_size:(k1 + group_size - 1) // group_size], k1 - k0, group_size)
        mk = m_all[:, k0:k1]
        for mv in np.unique(mk):
            if mv == 0:
                continue
            sel = np.where(mk == mv, x[:, k0:k1], 0.0).astype(np.float64)
            w = masked_codes(codes[k0:k1], np.full(k1 - k0, mv, dtype=np.uint8), max_bits).astype(np.float64)
            y += sel @ ((w + bias[mv]) * s)
    return y


def dense_weight(codes: np.ndarray, scales_f32: np.ndarray, group_size: int, dtype: str) -> np.ndarray:
    """``dtype(w * s)`` of the dense path (grinqh/kernel.py:586: ``w.to(dtype) * s``,
    rounded to the activation dtype), returned exactly as float32."""
    w = np.asarray(codes, dtype=np.float32)
    s = np.repeat(np.asarray(scales_f32, dtype=np.float32), group_size, axis=0)[: w.shape[0]]
    return to_f32(round_to_dtype(w * s, dtype), dtype)


def dense(x_f32: np.ndarray, codes: np.ndarray, scales_f32: np.ndarray,
          group_size: int, dtype: str) -> np.ndarray:
    """M > 1 dense path ``grinqh_prefill_gemm_compiled`` (grinqh/kernel.py:561-587):
    ``x @ dtype(w * s)`` -- the product is rounded to the activation dtype before
    the matmul (kernel.py:586); accumulation here is float64."""
    ws = dense_weight(codes, scales_f32, group_size, dtype).astype(np.float64)
    return np.asarray(x_f32, dtype=np.float64) @ ws


def gemm_or_gemv(x_f32, codes, scales_f32, bias_f32, max_bits, group_size, thresholds,
                 dtype: str, graded_prefill: bool = False):
    """Dispatch of ``torch.ops.grinqh.gemm_or_gemv`` (grinqh/kernel.py:646-710):
    rows > 1 -> dense (thresholds ignored, kernel.py:663-680); one row -> graded GEMV
    into fp32, cast, then bias add in the output dtype (kernel.py:706-708).
    ``graded_prefill`` selects this build's opt-in per-token grading for rows > 1.
    Returns the output in storage form of ``dtype``."""
    x = np.asarray(x_f32, dtype=np.float32).reshape(-1, np.asarray(x_f32).shape[-1])
    if x.shape[0] > 1 and not graded_prefill:
        y = round_to_dtype(dense(x, codes, scales_f32, group_size, dtype), dtype)
    else:
        y = round_to_dtype(looped_gemv(x, codes, scales_f32, thresholds, max_bits, group_size), dtype)
    if bias_f32 is not None:
        y = round_to_dtype(to_f32(y, dtype).astype(np.float64) + np.asarray(bias_f32, dtype=np.float32)[None, :], dtype)
    return y


# ----------------------------------------------------------------------------- checkpoint codec
def ct_pack_to_int32(codes: np.ndarray, num_bits: int) -> np.ndarray:
    """compressed-tensors ``pack_to_int32`` (packed_dim=1), the checkpoint format the
    loader reads (grinqh/grinqh.py:154-158): offset-binary ``code + 2^(b-1)``,
    ``32/b`` values per int32, LSB first along the last axis."""
    v = (np.asarray(codes, dtype=np.int16) + (1 << (num_bits - 1))).astype(np.uint32)
    rows, cols = v.shape
    pf = 32 // num_bits
    pad = (-cols) % pf
    if pad:
        v = np.pad(v, ((0, 0), (0, pad)))
    v = v.reshape(rows, -1, pf)
    out = np.zeros(v.shape[:2], dtype=np.uint32)
    for i in range(pf):
        out |= v[:, :, i] << np.uint32(i * num_bits)
    return out.view(np.int32)


def ct_unpack_from_int32(packed: np.ndarray, num_bits: int, shape) -> np.ndarray:
    """Inverse of :func:`ct_pack_to_int32` (compressed-tensors ``unpack_from_int32``)."""
    p = np.asarray(packed, dtype=np.int32).view(np.uint32)
    pf = 32 // num_bits
    mask = np.uint32((1 << num_bits) - 1)
    vals = np.stack([(p >> np.uint32(i * num_bits)) & mask for i in range(pf)], axis=-1)
    vals = vals.reshape(p.shape[0], -1)[:, : shape[1]].astype(np.int16) - (1 << (num_bits - 1))
    return vals.astype(np.int8)


# ----------------------------------------------------------------------------- synthetic data
def rtn_quantize(w_f32: np.ndarray, max_bits: int, group_size: int, dtype: str = "bf16"):
    """This build's synthetic quantizer (the reference ships none): symmetric
    round-to-nearest per (group_size-row K group, column),
    ``s = absmax / (2^(b-1)-1)`` stored in ``dtype``,
    ``code = clamp(rne(w / s), -2^(b-1), 2^(b-1)-1)``. ``w`` is (K, N)."""
    k, n = w_f32.shape
    qmax = (1 << (max_bits - 1)) - 1
    g = np.abs(w_f32.reshape(k // group_size, group_size, n)).max(axis=1)
    s_store = round_to_dtype(np.maximum(g / qmax, 1e-8), dtype)
    s = to_f32(s_store, dtype)
    q = np.rint(w_f32 / np.repeat(s, group_size, axis=0))
    codes = np.clip(q, -qmax - 1, qmax).astype(np.int8)
    return codes, s_store


def make_activations(rng: np.random.Generator, m: int, k: int, outlier_frac: float = 0.01,
                     outlier_scale: float = 20.0, outlier_idx=None, dist: str = "normal"):
    """N(0,1) activations with a fixed set of outlier channels scaled by 20
    (or unit-variance Student-t(3) when ``dist == 't3'``), float32."""
    if dist == "t3":
        x = rng.standard_t(3, size=(m, k)) / np.sqrt(3.0)
    else:
        x = rng.standard_normal((m, k))
    if outlier_idx is None:
        outlier_idx = np.sort(rng.choice(k, size=max(1, int(round(outlier_frac * k))), replace=False))
    if outlier_scale != 1.0:
        x[:, outlier_idx] *= outlier_scale
    return x.astype(np.float32), outlier_idx


def quantile_thresholds(abs_vals: np.ndarray, qs) -> list:
    """``torch.quantile`` (linear interpolation) of |x| at the given levels, as Python
    floats (tests/test_grinqh_ops.py:193-197)."""
    flat = np.sort(np.asarray(abs_vals, dtype=np.float32).reshape(-1).astype(np.float64))
    out = []
    for q in qs:
        pos = q * (flat.size - 1)
        lo = int(np.floor(pos))
        hi = min(lo + 1, flat.size - 1)
        frac = pos - lo
        out.append(float(np.float32(flat[lo] + (flat[hi] - flat[lo]) * frac)))
    return out
