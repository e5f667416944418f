"""Generate tests/golden/grinqh_golden.npz from the reference implementation itself.

Run once in a container where the reference project is importable (it is not
needed afterwards; the fixtures are committed):

    TRITON_INTERPRET=1 TORCHDYNAMO_DISABLE=1 \
        python tests/golden/make_golden.py --reference <path-to-vllm-grinqh-plugin>

What runs, all on CPU:
  * ``grinqh.utils._pack_kernel_uint32`` (the Triton pack kernel, utils.py:100-122)
    under the Triton interpreter, launched exactly as ``pack_triton`` launches it
    (utils.py:125-146; ``pack_triton`` itself asserts CUDA);
  * ``grinqh.utils.unpack_pyt`` (utils.py:149-177);
  * ``grinqh.kernel.grinqh_gemm_or_gemv`` (kernel.py:646-710; M==1 -> the Triton
    ``grinqh_gemv_uint32_packed`` under the interpreter, M>1 -> the dense path);
  * ``grinqh.kernel.grinqh_prefill_gemm_compiled`` eagerly (kernel.py:561-587);
  * ``grinqh.kernel.grinqh_gemv_batch_union`` (kernel.py:607-643, Triton interpreter);
  * ``compressed_tensors.pack_to_int32`` (the checkpoint codec the loader inverts).

Inputs are drawn from torch's CPU generator with fixed seeds and stored next to
the outputs, so the tests never depend on an RNG implementation.
bf16 tensors are stored as their uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")


def _store(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.uint32:
        return t.contiguous().view(torch.int32).numpy().view(np.uint32).copy()
    return t.contiguous().numpy().copy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "grinqh_golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    from grinqh import kernel as RK
    from grinqh import utils as RU
    from compressed_tensors import pack_to_int32

    def ref_pack(a_u32: torch.Tensor, max_bits: int) -> torch.Tensor:
        # pack_triton's host logic (utils.py:131-146) without its CUDA assert.
        a_u32 = a_u32.contiguous()
        m, n = a_u32.shape
        n_zone = n // 4
        n_out = n_zone * (max_bits // 2)
        out = torch.empty((m, n_out), dtype=a_u32.dtype)
        RU._pack_kernel_uint32[(m, -(-n_out // 256))](
            a_u32, out, a_u32.stride(0), a_u32.stride(1), n_zone, n_out, BLOCK=256)
        return out

    def packed_from_codes(w_i8: torch.Tensor, max_bits: int) -> torch.Tensor:
        # process_weights_after_loading (grinqh.py:202-211)
        shuffled = RU.grinqh_input_preshuffle(w_i8)
        shifted = shuffled << (8 - max_bits)
        return ref_pack(shifted.view(torch.uint32), max_bits)

    dt = {"bf16": torch.bfloat16, "f16": torch.float16}
    g = {}

    # ---- pack / unpack (tests/test_grinqh_ops.py:58-88 shapes) -------------------------
    torch.manual_seed(1)
    a = torch.randint(0, 256, (384, 320), dtype=torch.uint8)
    g["pack_in_u8"] = _store(a)
    for b in (2, 4, 6, 8):
        p = ref_pack(a.view(torch.uint32), b)
        g[f"pack_out_b{b}"] = _store(p)
        rec = RU.unpack_pyt(p, torch.arange(384), RU.BitLevel(b // 2), original_n=a.view(torch.uint32).shape[1])
        g[f"unpack_out_b{b}"] = rec.view(torch.uint8).numpy().copy()

    # ---- codes per bit width (shared by GEMV / dense cases) ------------------------------
    K, N, G = 256, 256, 128
    for b in (2, 4, 6, 8):
        torch.manual_seed(10 + b)
        lim = (1 << (b - 1)) - 1
        w = torch.randint(-lim - 1, lim + 1, (K, N), dtype=torch.int8)
        g[f"codes_b{b}"] = w.numpy().copy()
        g[f"packed_b{b}"] = _store(packed_from_codes(w, b))

    # ---- graded M==1 GEMV (tests/test_grinqh_ops.py:156-240) -----------------------------
    qsets = {
        "spread": [0.2, 0.4, 0.6, 0.8], "all_or_nothing": [0.5] * 4, "mild": [0.1, 0.2, 0.3, 0.4],
        "aggressive": [0.6, 0.7, 0.8, 0.9], "skip_all": [1.0] * 4, "dense": None,
    }
    for dname, dtype in dt.items():
        torch.manual_seed(100 + len(dname))
        x = torch.randn((1, K), dtype=dtype)
        s = torch.randn((K // G, N), dtype=dtype)
        g[f"gemv_x_{dname}"] = _store(x)
        g[f"gemv_s_{dname}"] = _store(s)
        for b in (2, 4, 6, 8):
            packed = torch.from_numpy(g[f"packed_b{b}"].view(np.int32)).view(torch.uint32)
            nz = b // 2
            for qname, qs in qsets.items():
                if qs is None:
                    th = [-1.0] * 4
                else:
                    th = torch.quantile(x.abs().float(), torch.tensor(qs))[:nz].tolist()
                    th = th + [0.0] * (4 - nz)
                y = RK.grinqh_gemm_or_gemv(x=x, weight_packed=packed, weight_scale=s, bias=None,
                                           max_bits=b, group_size=G, original_n=N // 4, thresholds=th)
                key = f"gemv_{dname}_b{b}_{qname}"
                g[key + "_th"] = np.array(th, dtype=np.float64)
                g[key + "_y"] = _store(y)

    # ---- batch-union GEMV (tests/test_grinqh_ops.py:245-282) + graded union ---------------
    for dname in ("bf16", "f16"):
        for bs in (2, 3, 5, 8):
            torch.manual_seed(200 + bs)
            x = torch.randn((bs, K), dtype=dt[dname])
            s = torch.randn((K // G, N), dtype=dt[dname])
            g[f"union_x_{dname}_m{bs}"] = _store(x)
            g[f"union_s_{dname}_m{bs}"] = _store(s)
            for b in (2, 4, 6, 8):
                packed = torch.from_numpy(g[f"packed_b{b}"].view(np.int32)).view(torch.uint32)
                for tname in ("dense", "spread"):
                    if tname == "dense":
                        th = [-1.0] * 4
                    else:
                        th = torch.quantile(x.abs().amax(0).float(), torch.tensor([0.2, 0.4, 0.6, 0.8]))[: b // 2].tolist()
                        th = th + [0.0] * (4 - b // 2)
                    y = RK.grinqh_gemv_batch_union(x=x, weight_packed=packed, weight_scale=s, bias=None,
                                                   max_bits=b, group_size=G, original_n=N // 4, thresholds=th)
                    key = f"union_{dname}_m{bs}_b{b}_{tname}"
                    g[key + "_th"] = np.array(th, dtype=np.float64)
                    g[key + "_y"] = _store(y)

    # ---- dense M>1 path (tests/test_grinqh_ops.py:91-124 shapes: 16 x 384 x 320) ----------
    Kd, Nd = 384, 320
    for b in (2, 4, 6, 8):
        torch.manual_seed(300 + b)
        lim = (1 << (b - 1)) - 1
        w = torch.randint(-lim - 1, lim + 1, (Kd, Nd), dtype=torch.int8)
        g[f"dense_codes_b{b}"] = w.numpy().copy()
        packed = packed_from_codes(w, b)
        g[f"dense_packed_b{b}"] = _store(packed)
        for dname, dtype in dt.items():
            x = torch.randn((16, Kd), dtype=dtype)
            s = torch.randn((Kd // G, Nd), dtype=dtype)
            y = RK.grinqh_prefill_gemm_compiled(x, packed, s, G, Nd // 4, b)
            key = f"dense_{dname}_b{b}"
            g[key + "_x"] = _store(x)
            g[key + "_s"] = _store(s)
            g[key + "_y"] = _store(y)

    # ---- op with bias: M==1 graded and M==4 dense (kernel.py:706-710) ----------------------
    torch.manual_seed(400)
    for dname, dtype in dt.items():
        for rows in (1, 4):
            x = torch.randn((rows, K), dtype=dtype)
            s = torch.randn((K // G, N), dtype=dtype) * 0.05
            bias = torch.randn((N,), dtype=dtype)
            packed = torch.from_numpy(g["packed_b8"].view(np.int32)).view(torch.uint32)
            th = torch.quantile(x.abs().float(), torch.tensor([0.2, 0.4, 0.6, 0.8])).tolist()
            y = RK.grinqh_gemm_or_gemv(x=x, weight_packed=packed, weight_scale=s, bias=bias,
                                       max_bits=8, group_size=G, original_n=N // 4, thresholds=th)
            key = f"bias_{dname}_m{rows}"
            g[key + "_x"], g[key + "_s"], g[key + "_bias"] = _store(x), _store(s), _store(bias)
            g[key + "_th"] = np.array(th, dtype=np.float64)
            g[key + "_y"] = _store(y)

    # ---- a config-like case: RTN-quantized N(0, 0.02) weights, outlier activations ----------
    Kc, Nc = 512, 256
    torch.manual_seed(500)
    wf = torch.randn((Kc, Nc)) * 0.02
    qmax = 127
    sc = (wf.view(Kc // G, G, Nc).abs().amax(1) / qmax).to(torch.bfloat16)
    codes = torch.clamp(torch.round(wf / sc.float().repeat_interleave(G, 0)), -128, 127).to(torch.int8)
    xc = torch.randn((1, Kc))
    out_idx = torch.randperm(Kc)[: Kc // 100]
    xc[:, out_idx] *= 20
    xc = xc.to(torch.bfloat16)
    th = torch.quantile(xc.abs().float(), torch.tensor([0.2, 0.4, 0.6, 0.8])).tolist()
    packed = packed_from_codes(codes, 8)
    y = RK.grinqh_gemm_or_gemv(x=xc, weight_packed=packed, weight_scale=sc, bias=None,
                               max_bits=8, group_size=G, original_n=Nc // 4, thresholds=th)
    g["cfg_codes"], g["cfg_s"], g["cfg_x"] = codes.numpy().copy(), _store(sc), _store(xc)
    g["cfg_packed"], g["cfg_th"], g["cfg_y"] = _store(packed), np.array(th), _store(y)

    # ---- compressed-tensors checkpoint codec (loader input, grinqh.py:154-158) --------------
    for b in (2, 4, 6, 8):
        torch.manual_seed(600 + b)
        lim = (1 << (b - 1)) - 1
        w = torch.randint(-lim - 1, lim + 1, (64, 256), dtype=torch.int8)  # (N, K) checkpoint orientation
        g[f"ct_codes_b{b}"] = w.numpy().copy()
        g[f"ct_packed_b{b}"] = pack_to_int32(w, b).numpy().copy()

    np.savez_compressed(args.out, **g)
    print(f"wrote {args.out}: {len(g)} arrays, {os.path.getsize(args.out) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
