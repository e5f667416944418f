"""grinqh_gemv_noalloc: the single-row graded GEMV for callers that cannot allocate
device memory while they run (fixed start-up memory budgets, allocation-free hot
paths). It keeps its scratch in a fixed array inside the library; this checks,
through the C ABI, that two calls in a row match the workspace-taking entry point
and that bad arguments are refused. Collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _problem(K, N, seed):
    from grinqh.utils import pack_codes
    g = torch.Generator(device="cuda").manual_seed(seed)
    codes = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    w = pack_codes(codes, 8)
    s = (torch.rand((K // 128, N), device="cuda", generator=g) * 1e-2).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    return w, s, bias


@pytest.mark.parametrize("K,N", [(14336, 4096), (4096, 6144), (256, 256)])
def test_noalloc_matches_workspace_entry_point_twice(K, N):
    from grinqh import _ext
    lib = _ext.cabi()
    w, s, bias = _problem(K, N, K + N)
    th = _ext.thresholds_arg([0.3, 0.6, 1.0, 1.5])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws_bytes = lib.grinqh_workspace_size(1, K, N, 8, 128, _ext.MODE_AUTO)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    for call in range(2):  # the second call checks what the first one left behind
        x = torch.randn(1, K, device="cuda").to(torch.bfloat16) * (1 + call)
        y_ref = torch.empty(1, N, dtype=torch.bfloat16, device="cuda")
        y = torch.full((1, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.grinqh_gemm_or_gemv(_ptr(x), _ext.GRINQH_BF16, 1, K, _ptr(w), _ptr(s), _ptr(bias), 8, 128, N, th,
                                     _ext.MODE_AUTO, _ptr(y_ref), _ptr(ws), ws_bytes, stream)
        assert st == 0, lib.grinqh_last_error()
        st = lib.grinqh_gemv_noalloc(_ptr(x), _ext.GRINQH_BF16, K, _ptr(w), _ptr(s), _ptr(bias), 8, 128, N, th,
                                     _ptr(y), stream)
        assert st == 0, lib.grinqh_last_error()
        torch.cuda.synchronize()
        a, b = y.float().cpu().numpy(), y_ref.float().cpu().numpy()
        assert np.isfinite(a).all()
        err = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
        fro = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert err <= 1e-2 and fro <= 2e-3, (call, err, fro)


def test_noalloc_refuses_bad_arguments():
    from grinqh import _ext
    lib = _ext.cabi()
    dummy = torch.zeros(64, dtype=torch.int32, device="cuda")
    th = _ext.thresholds_arg([0.0] * 4)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # N not a multiple of 16 (the packed layout needs N % 16 == 0)
    st = lib.grinqh_gemv_noalloc(_ptr(dummy), _ext.GRINQH_BF16, 256, _ptr(dummy), _ptr(dummy), None, 8, 128, 40,
                                 th, _ptr(dummy), stream)
    assert st == 1 and b"multiple of 16" in lib.grinqh_last_error()
    # unsupported bit width
    st = lib.grinqh_gemv_noalloc(_ptr(dummy), _ext.GRINQH_BF16, 256, _ptr(dummy), _ptr(dummy), None, 3, 128, 64,
                                 th, _ptr(dummy), stream)
    assert st == 2
