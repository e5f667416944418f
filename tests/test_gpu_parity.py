"""GPU parity of the sm_100a kernels, called through the torch ops (which call the
C ABI): bit-exact pack / unpack / grade, and linear outputs against the reference's
own kernel outputs (tests/golden) and against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import FRO_TOL, MAX_REL_TOL, rel_errors

pytestmark = pytest.mark.gpu

BITS = (2, 4, 6, 8)
DTYPES = ("bf16", "f16")
TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import grinqh.kernel  # noqa: F401


def dev_act(a, dtype):
    """storage form (uint16 bits for bf16, float16) -> CUDA tensor of dtype."""
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).cuda()


def dev_words(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).cuda()


def host_words(t):
    return t.cpu().contiguous().view(torch.int32).numpy().view(np.uint32)


def f32(t):
    return t.float().cpu().numpy()


@pytest.fixture(params=["streaming", "tensor_cores"])
def m1_kernel(request, monkeypatch):
    """Runs a single-row test on both single-row kernels: the default register-
    streaming one and the opt-in int8 tensor-core one (GRINQH_M1_TENSOR_CORES=1)."""
    if request.param == "tensor_cores":
        monkeypatch.setenv("GRINQH_M1_TENSOR_CORES", "1")
    else:
        monkeypatch.delenv("GRINQH_M1_TENSOR_CORES", raising=False)
    return request.param


def assert_parity(got, ref, max_rel=MAX_REL_TOL, fro=FRO_TOL):
    mx, fr = rel_errors(got, ref)
    assert mx <= max_rel and fr <= fro, f"max-rel {mx:.3e} (<= {max_rel}), fro {fr:.3e} (<= {fro})"


# ----------------------------------------------------------------------------- codec
@pytest.mark.parametrize("b", BITS)
def test_pack_words_matches_reference_kernel(golden, b):
    from grinqh.utils import pack_triton
    a = torch.from_numpy(golden["pack_in_u8"]).cuda()
    out = pack_triton(a.view(torch.uint32), max_bits=b)
    np.testing.assert_array_equal(host_words(out), golden[f"pack_out_b{b}"])
    assert out.numel() * out.element_size() == a.numel() * b // 8


@pytest.mark.parametrize("b", BITS)
def test_unpack_matches_reference(golden, b):
    from grinqh.utils import BitLevel, unpack_pyt, unpack_triton
    packed = dev_words(golden[f"pack_out_b{b}"]).view(torch.uint32)
    k = packed.shape[0]
    orig_n = golden["pack_in_u8"].shape[1] // 4
    rec = unpack_pyt(packed, torch.arange(k), BitLevel(b // 2), original_n=orig_n).view(torch.uint8)
    np.testing.assert_array_equal(rec.cpu().numpy(), golden[f"unpack_out_b{b}"])
    row = unpack_triton(packed, 5, BitLevel(b // 2), original_n=orig_n).view(torch.uint8)
    np.testing.assert_array_equal(row.cpu().numpy(), golden[f"unpack_out_b{b}"][5])


@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("shape", [(256, 256), (384, 320), (128, 16), (96, 4112)])
def test_pack_codes_bit_exact(golden, b, shape):
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(b * 100 + shape[1])
    lim = 1 << (b - 1)
    codes = rng.integers(-lim, lim, size=shape).astype(np.int8)
    out = pack_codes(torch.from_numpy(codes).cuda(), b)
    np.testing.assert_array_equal(host_words(out), O.pack_codes(codes, b))


@pytest.mark.parametrize("b", BITS)
def test_pack_codes_matches_reference_layout(golden, b):
    from grinqh.utils import pack_codes
    out = pack_codes(torch.from_numpy(golden[f"codes_b{b}"]).cuda(), b)
    np.testing.assert_array_equal(host_words(out), golden[f"packed_b{b}"])
    out = pack_codes(torch.from_numpy(golden[f"dense_codes_b{b}"]).cuda(), b)
    np.testing.assert_array_equal(host_words(out), golden[f"dense_packed_b{b}"])


def test_pack_codes_strided_rows():
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(5)
    big = rng.integers(-128, 128, size=(64, 96)).astype(np.int8)
    t = torch.from_numpy(big).cuda()[:, :64]  # row stride 96
    np.testing.assert_array_equal(host_words(pack_codes(t, 8)), O.pack_codes(big[:, :64], 8))


# ----------------------------------------------------------------------------- grade
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
def test_grade_bit_exact(dtype, b):
    from grinqh.kernel import grinqh_grade
    rng = np.random.default_rng(11 + b)
    x = rng.standard_normal((5, 1000)).astype(np.float32)
    xs = O.round_to_dtype(x, dtype)
    x32 = O.to_f32(xs, dtype)
    # thresholds equal to element values exercise the strict '>' boundary
    th = [float(np.abs(x32[0, 3])), float(np.abs(x32[1, 7])), 0.5, float(np.abs(x32[2, 9]))]
    masks, uni = grinqh_grade(dev_act(xs, dtype), th, b)
    exp = O.grade(x32, th, b)
    np.testing.assert_array_equal(masks.cpu().numpy(), exp)
    np.testing.assert_array_equal(uni.cpu().numpy(), np.bitwise_or.reduce(exp, axis=0))


# ----------------------------------------------------------------------------- linear vs reference outputs
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("q", ["spread", "all_or_nothing", "mild", "aggressive", "skip_all", "dense"])
def test_graded_gemv_matches_reference(golden, dtype, b, q, m1_kernel):
    """M == 1 graded GEMV vs the reference Triton kernel's output on identical inputs
    (tests/test_grinqh_ops.py:156-240 cases)."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    key = f"gemv_{dtype}_b{b}_{q}"
    x = dev_act(golden[f"gemv_x_{dtype}"], dtype)
    s = dev_act(golden[f"gemv_s_{dtype}"], dtype)
    w = dev_words(golden[f"packed_b{b}"])
    th = golden[key + "_th"].tolist()
    y = grinqh_gemm_or_gemv(x, w, s, None, b, 128, 64, th)
    ref = O.to_f32(golden[key + "_y"], dtype)
    got = f32(y)
    if q == "skip_all":
        assert np.count_nonzero(got) == 0 and np.count_nonzero(ref) == 0
        return
    assert_parity(got, ref)
    torch.testing.assert_close(y, torch.from_numpy(ref).to(TDT[dtype]).cuda())
    # and against the oracle
    y_or = O.graded_gemv(O.to_f32(golden[f"gemv_x_{dtype}"], dtype)[0], golden[f"codes_b{b}"],
                         O.to_f32(golden[f"gemv_s_{dtype}"], dtype), th, b, 128)
    assert_parity(got[0], O.to_f32(O.round_to_dtype(y_or, dtype), dtype))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
@pytest.mark.parametrize("m", [2, 3, 5, 8])
@pytest.mark.parametrize("t", ["dense", "spread"])
def test_batch_union_matches_reference(golden, dtype, b, m, t):
    from grinqh.kernel import grinqh_gemv_batch_union
    key = f"union_{dtype}_m{m}_b{b}_{t}"
    x = dev_act(golden[f"union_x_{dtype}_m{m}"], dtype)
    s = dev_act(golden[f"union_s_{dtype}_m{m}"], dtype)
    y = grinqh_gemv_batch_union(x, dev_words(golden[f"packed_b{b}"]), s, None, b, 128, 64,
                                golden[key + "_th"].tolist())
    ref = O.to_f32(golden[key + "_y"], dtype)
    assert_parity(f32(y), ref)
    torch.testing.assert_close(y, torch.from_numpy(ref).to(TDT[dtype]).cuda(), atol=1e-3, rtol=1.6e-2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", BITS)
def test_dense_matches_reference(golden, dtype, b):
    """M > 1 dense path vs the reference's grinqh_prefill_gemm_compiled on identical
    inputs (tests/test_grinqh_ops.py:91-124 shapes, 16 x 384 x 320)."""
    from grinqh.kernel import grinqh_gemm_or_gemv, grinqh_prefill_gemm_compiled
    key = f"dense_{dtype}_b{b}"
    x = dev_act(golden[key + "_x"], dtype)
    s = dev_act(golden[key + "_s"], dtype)
    w = dev_words(golden[f"dense_packed_b{b}"])
    ref = O.to_f32(golden[key + "_y"], dtype)
    y1 = grinqh_prefill_gemm_compiled(x, w, s, 128, 80, b)
    y2 = grinqh_gemm_or_gemv(x, w, s, None, b, 128, 80, [0.3] * 4)  # rows > 1 -> dense, thresholds ignored
    for y in (y1, y2):
        assert_parity(f32(y), ref)
        # the golden output came from the CPU matmul: fp32 summation order differs, so an
        # element near cancellation may land 1-2 fp16 ulp away (torch's fp16 default
        # rtol=1e-3 is tighter than 2 ulp); bf16 keeps torch's defaults
        tol = dict(rtol=4e-3, atol=1e-3) if dtype == "f16" else {}
        torch.testing.assert_close(y, torch.from_numpy(ref).to(TDT[dtype]).cuda(), **tol)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows", [1, 4])
def test_bias_matches_reference(golden, dtype, rows):
    from grinqh.kernel import grinqh_gemm_or_gemv
    key = f"bias_{dtype}_m{rows}"
    y = grinqh_gemm_or_gemv(dev_act(golden[key + "_x"], dtype), dev_words(golden["packed_b8"]),
                            dev_act(golden[key + "_s"], dtype), dev_act(golden[key + "_bias"], dtype),
                            8, 128, 64, golden[key + "_th"].tolist())
    assert_parity(f32(y), O.to_f32(golden[key + "_y"], dtype))


def test_config_like_case_matches_reference(golden):
    from grinqh.kernel import grinqh_gemm_or_gemv
    y = grinqh_gemm_or_gemv(dev_act(golden["cfg_x"], "bf16"), dev_words(golden["cfg_packed"]),
                            dev_act(golden["cfg_s"], "bf16"), None, 8, 128, 64, golden["cfg_th"].tolist())
    assert_parity(f32(y), O.to_f32(golden["cfg_y"], "bf16"))


# ----------------------------------------------------------------------------- larger shapes vs oracle
def _problem(rng, K, N, b, M, dtype="bf16", dist="normal"):
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    codes, s_store = O.rtn_quantize(w, b, 128, dtype)
    x, _ = O.make_activations(rng, M, K, dist=dist)
    xs = O.round_to_dtype(x, dtype)
    x32 = O.to_f32(xs, dtype)
    cal, _ = O.make_activations(rng, 64, K)
    th = O.quantile_thresholds(np.abs(O.to_f32(O.round_to_dtype(cal, dtype), dtype)), [0.2, 0.4, 0.6, 0.8])
    return codes, s_store, xs, x32, th


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 6144), (14336, 4096)])
@pytest.mark.parametrize("b", [8, 4])
def test_llama_shapes_graded_m1(K, N, b, m1_kernel):
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(K + N + b)
    codes, s_store, xs, x32, th = _problem(rng, K, N, b, 1)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, "bf16"), w, dev_act(s_store, "bf16"), None, b, 128, N // 4, th)
    ref = O.graded_gemv(x32[0], codes, O.to_f32(s_store, "bf16"), th, b, 128)
    assert_parity(f32(y)[0], O.to_f32(O.round_to_dtype(ref, "bf16"), "bf16"))


@pytest.mark.parametrize("K,N", [(512, 4128), (384, 4112), (1024, 96), (256, 1056), (512, 4160), (1024, 64),
                                 (384, 1088), (4096, 9216)])
@pytest.mark.parametrize("b", [8, 6, 2])
def test_ragged_widths_graded_m1(K, N, b, m1_kernel):
    """Widths the single-row kernel slices unevenly: a partial last 1024-column slice
    (N = 4128, 1056, 4160, 1088, 9216), less than one slice (96, 64); N / 16 odd (4112)
    runs the generic kernel."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(K * 7 + N + b)
    codes, s_store, xs, x32, th = _problem(rng, K, N, b, 1)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, "bf16"), w, dev_act(s_store, "bf16"), None, b, 128, N // 4, th)
    ref = O.graded_gemv(x32[0], codes, O.to_f32(s_store, "bf16"), th, b, 128)
    assert_parity(f32(y)[0], O.to_f32(O.round_to_dtype(ref, "bf16"), "bf16"))


@pytest.mark.parametrize("M", [2, 16, 33])
@pytest.mark.parametrize("b", [8, 4])
def test_llama_shape_dense_small_m(M, b):
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    K, N = 4096, 4096
    rng = np.random.default_rng(M * 7 + b)
    codes, s_store, xs, x32, th = _problem(rng, K, N, b, M)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, "bf16"), w, dev_act(s_store, "bf16"), None, b, 128, N // 4, th)
    ref = O.dense(x32, codes, O.to_f32(s_store, "bf16"), 128, "bf16")
    assert_parity(f32(y), O.to_f32(O.round_to_dtype(ref, "bf16"), "bf16"))


@pytest.mark.parametrize("M", [3, 8])
def test_graded_rows_equal_looped_gemv(M):
    """MODE_GRADED grades every row by itself: same as calling the M==1 path per row."""
    from grinqh.kernel import MODE_GRADED, grinqh_gemm_or_gemv, grinqh_linear
    from grinqh.utils import pack_codes
    K, N, b = 1024, 512, 8
    rng = np.random.default_rng(M)
    codes, s_store, xs, x32, th = _problem(rng, K, N, b, M)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    s = dev_act(s_store, "bf16")
    x = dev_act(xs, "bf16")
    y = grinqh_linear(x, w, s, None, b, 128, N // 4, th, MODE_GRADED)
    loop = torch.cat([grinqh_gemm_or_gemv(x[i:i + 1], w, s, None, b, 128, N // 4, th) for i in range(M)])
    assert_parity(f32(y), f32(loop), max_rel=4e-3, fro=1e-3)
    ref = O.looped_gemv(x32, codes, O.to_f32(s_store, "bf16"), th, b, 128)
    assert_parity(f32(y), O.to_f32(O.round_to_dtype(ref, "bf16"), "bf16"))


# ----------------------------------------------------------------------------- edge cases and properties
def test_empty_rows_and_3d_input():
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(1)
    codes = rng.integers(-128, 128, size=(256, 64)).astype(np.int8)
    w = pack_codes(torch.from_numpy(codes).cuda(), 8)
    s = torch.rand(2, 64, dtype=torch.bfloat16, device="cuda")
    y0 = grinqh_gemm_or_gemv(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda"), w, s, None, 8, 128, 16, [0.0] * 4)
    assert y0.shape == (0, 64)
    x3 = torch.randn(2, 3, 256, dtype=torch.bfloat16, device="cuda")
    y3 = grinqh_gemm_or_gemv(x3, w, s, None, 8, 128, 16, [0.0] * 4)
    y2 = grinqh_gemm_or_gemv(x3.reshape(6, 256), w, s, None, 8, 128, 16, [0.0] * 4)
    assert y3.shape == (2, 3, 64)
    assert torch.equal(y3.reshape(6, 64), y2)
    xt = torch.randn(256, 1, dtype=torch.bfloat16, device="cuda").t()  # non-contiguous view
    assert torch.equal(grinqh_gemm_or_gemv(xt, w, s, None, 8, 128, 16, [0.1] * 4),
                       grinqh_gemm_or_gemv(xt.contiguous(), w, s, None, 8, 128, 16, [0.1] * 4))


def test_invalid_arguments_raise():
    from grinqh.kernel import grinqh_gemm_or_gemv
    w = torch.zeros(256, 4 * 4, dtype=torch.int32, device="cuda")
    s = torch.ones(2, 64, dtype=torch.bfloat16, device="cuda")
    x = torch.randn(1, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="max_bits"):
        grinqh_gemm_or_gemv(x, w, s, None, 3, 128, 16, [0.0] * 4)
    with pytest.raises(RuntimeError, match="x.shape"):
        grinqh_gemm_or_gemv(x[:, :128], w, s, None, 8, 128, 16, [0.0] * 4)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        grinqh_gemm_or_gemv(x.float(), w, s, None, 8, 128, 16, [0.0] * 4)
    with pytest.raises(RuntimeError, match="weight_scale"):
        grinqh_gemm_or_gemv(x, w, s[:1], None, 8, 128, 16, [0.0] * 4)


@pytest.mark.parametrize("M", [1, 16])
def test_scaling_and_determinism_at_full_size(M):
    """Size-independent properties at the gate_up shape (K=4096, N=28672): power-of-two
    scaling of x (and thresholds) scales y exactly; repeated calls are bit-identical;
    thresholds above every |x| read no plane and give exactly zero."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    K, N, b = 4096, 28672, 8
    rng = np.random.default_rng(42)
    codes = rng.integers(-128, 128, size=(K, N)).astype(np.int8)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    s = (torch.rand(K // 128, N, device="cuda") * 1e-3).to(torch.bfloat16)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    th = [0.3, 0.6, 1.0, 1.5]
    y = grinqh_gemm_or_gemv(x, w, s, None, b, 128, N // 4, th)
    y_again = grinqh_gemm_or_gemv(x, w, s, None, b, 128, N // 4, th)
    assert torch.equal(y, y_again)
    y4 = grinqh_gemm_or_gemv(x * 4, w, s, None, b, 128, N // 4, [4 * t for t in th])
    assert torch.equal(y4, y * 4)
    if M == 1:
        z = grinqh_gemm_or_gemv(x, w, s, None, b, 128, N // 4, [1e30] * 4)
        assert torch.count_nonzero(z) == 0


def test_no_pipeline_wait_timed_out():
    """Every bounded mbarrier wait in the kernels run so far completed in time."""
    import ctypes
    from grinqh import _ext
    v = ctypes.c_uint(123)
    assert _ext.cabi().grinqh_take_error_flags(ctypes.byref(v)) == 0
    assert v.value == 0


@pytest.mark.parametrize("M,K,N", [(64, 256, 256), (300, 384, 320), (512, 1024, 4096), (256, 4096, 6144)])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", [8, 4, 2, 6])
def test_dense_tensor_core_gemm(M, K, N, dtype, b):
    """Rows >= 64 run the tcgen05 GEMM (in-kernel dequant to dtype(w*s)); vs the oracle,
    including a row tail (300), a column tail (N/16 = 20 words) and multiple tiles."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(M + K + N + b)
    lim = 1 << (b - 1)
    codes = rng.integers(-lim, lim, size=(K, N)).astype(np.int8)
    s32 = (rng.random((K // 128, N)) * 0.02 + 0.001).astype(np.float32)
    s_store = O.round_to_dtype(s32, dtype)
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs = O.round_to_dtype(x, dtype)
    bias = O.round_to_dtype(rng.standard_normal(N).astype(np.float32), dtype)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128,
                            N // 4, [0.0] * 4)
    ref = O.gemm_or_gemv(O.to_f32(xs, dtype), codes, O.to_f32(s_store, dtype), O.to_f32(bias, dtype), b, 128,
                         [0.0] * 4, dtype)
    assert_parity(f32(y), O.to_f32(ref, dtype))


@pytest.mark.parametrize("M,K,N", [(2, 256, 256), (5, 384, 320), (16, 4096, 1024), (17, 1024, 4128),
                                   (33, 2048, 6144), (48, 512, 544), (64, 8192, 512), (17, 1024, 4112),
                                   (48, 512, 528)])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", [8, 4, 2, 6])
def test_dense_skinny_gemm(M, K, N, dtype, b):
    """Rows 2..64 run the skinny tcgen05 GEMM (weights as operand A, tokens as N): a
    single cluster (2 x 256 x 256, 5 x 384 x 320), several clusters per tile
    (16 x 4096 x 1024: 64 splits in clusters of 8), partial column tiles (N/16 = 258,
    34), padded token counts (17, 33, 48) and the largest count (64). N/16 odd (4112,
    528) falls back to the generic kernel."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(M * 31 + K + N + b)
    lim = 1 << (b - 1)
    codes = rng.integers(-lim, lim, size=(K, N)).astype(np.int8)
    s32 = (rng.random((K // 128, N)) * 0.02 + 0.001).astype(np.float32)
    s_store = O.round_to_dtype(s32, dtype)
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs = O.round_to_dtype(x, dtype)
    bias = O.round_to_dtype(rng.standard_normal(N).astype(np.float32), dtype)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128,
                            N // 4, [0.0] * 4)
    ref = O.gemm_or_gemv(O.to_f32(xs, dtype), codes, O.to_f32(s_store, dtype), O.to_f32(bias, dtype), b, 128,
                         [0.0] * 4, dtype)
    assert_parity(f32(y), O.to_f32(ref, dtype))
    y2 = grinqh_gemm_or_gemv(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128,
                             N // 4, [0.0] * 4)
    assert torch.equal(y, y2), "skinny GEMM is not deterministic"


@pytest.mark.parametrize("M,K,N", [(512, 256, 4128), (600, 384, 320), (1024, 1024, 1024), (520, 256, 4112),
                                   (128, 14336, 1024), (200, 4096, 2048), (65, 2048, 1056)])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", [8, 4, 2, 6])
def test_dense_two_pass_gemm(M, K, N, dtype, b):
    """Rows >= 512 (or few output tiles) dequantize once to dtype(w*s) and run the
    TMA-fed tcgen05 GEMM: a partial last column tile (N = 4128), a row tail (600) and
    several tiles each way; N/16 odd (4112) takes the fused GEMM instead. Few output
    tiles split K over the SMs (1024^3, 128 x 14336 x 1024, 200 rows, 65 rows with a
    partial column tile), the splits added in order by the last one."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(M + 3 * K + N + b)
    lim = 1 << (b - 1)
    codes = rng.integers(-lim, lim, size=(K, N)).astype(np.int8)
    s32 = (rng.random((K // 128, N)) * 0.02 + 0.001).astype(np.float32)
    s_store = O.round_to_dtype(s32, dtype)
    x = rng.standard_normal((M, K)).astype(np.float32)
    xs = O.round_to_dtype(x, dtype)
    bias = O.round_to_dtype(rng.standard_normal(N).astype(np.float32), dtype)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_gemm_or_gemv(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128,
                            N // 4, [0.0] * 4)
    ref = O.gemm_or_gemv(O.to_f32(xs, dtype), codes, O.to_f32(s_store, dtype), O.to_f32(bias, dtype), b, 128,
                         [0.0] * 4, dtype)
    assert_parity(f32(y), O.to_f32(ref, dtype))
    y2 = grinqh_gemm_or_gemv(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128,
                             N // 4, [0.0] * 4)
    assert torch.equal(y, y2), "two-pass GEMM is not deterministic"


@pytest.mark.parametrize("M,K,N", [(128, 1024, 512), (300, 512, 1056), (256, 384, 4096)])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b", [8, 6, 4, 2])
@pytest.mark.parametrize("q", ["spread", "non_monotone"])
def test_graded_prefill_tensor_cores(M, K, N, dtype, b, q):
    """MODE_GRADED with 128 rows or more runs the tensor-core graded prefill: one fp16 GEMM
    over the zone-masked activations and the zone weight operands (bias folded in). Against
    the oracle's per-token grading (grinqh/kernel.py:100-158 applied row by row), with a
    row tail (300 rows), a partial column tile (1056), non-monotone thresholds (masks
    with gaps), bias, and a block of rows whose activations are all zero (skipped steps)."""
    from grinqh.kernel import MODE_GRADED, grinqh_linear
    from grinqh.utils import pack_codes
    rng = np.random.default_rng(M + K + N + b + len(q))
    lim = 1 << (b - 1)
    codes = rng.integers(-lim, lim, size=(K, N)).astype(np.int8)
    s32 = (rng.random((K // 128, N)) * 0.02 + 0.001).astype(np.float32)
    s_store = O.round_to_dtype(s32, dtype)
    x, _ = O.make_activations(rng, M, K, dist="t3")
    x[: min(M, 256) // 2, : K // 2] = 0.0  # a zero block: its steps have no active value
    xs = O.round_to_dtype(x, dtype)
    x32 = O.to_f32(xs, dtype)
    ax = np.abs(x32[np.abs(x32) > 0])
    qs = [0.2, 0.4, 0.6, 0.8] if q == "spread" else [0.5, 0.1, 0.9, 0.3]
    th = O.quantile_thresholds(ax, qs)
    bias = O.round_to_dtype(rng.standard_normal(N).astype(np.float32), dtype)
    w = pack_codes(torch.from_numpy(codes).cuda(), b)
    y = grinqh_linear(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128, N // 4, th,
                      MODE_GRADED)
    # the op's result: the graded rows rounded to dtype, then the bias added in dtype
    # (grinqh/kernel.py:706-708), as oracle.gemm_or_gemv(graded_prefill=True) computes it
    yr = O.to_f32(O.round_to_dtype(O.graded_rows(x32, codes, O.to_f32(s_store, dtype), th, b, 128), dtype), dtype)
    ref = O.to_f32(O.round_to_dtype(yr.astype(np.float64) + O.to_f32(bias, dtype)[None, :], dtype), dtype)
    assert_parity(f32(y), ref)
    y2 = grinqh_linear(dev_act(xs, dtype), w, dev_act(s_store, dtype), dev_act(bias, dtype), b, 128, N // 4, th,
                       MODE_GRADED)
    assert torch.equal(y, y2), "graded prefill is not deterministic"
