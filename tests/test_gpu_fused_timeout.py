"""The fused row-parallel kernels' bounded wait (the single-row GEMV and the skinny
GEMM of 2..64 rows), on one GPU, without a fault or a hang: a launch as rank 0 of 2
ranks whose second rank is a zeroed local buffer that nobody writes. Its wait for rank 1's partials must run out after the short limit set by
GRINQH_ALLREDUCE_WAIT_MS, the kernel must return, grinqh_take_error_flags must report
it (and clear it), and the next launch -- a single-rank one on the same buffer -- must
be correct again."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _take():
    from grinqh._ext import cabi
    n = ctypes.c_uint(0)
    assert cabi().grinqh_take_error_flags(ctypes.byref(n)) == 0
    return n.value


def _alloc(lib, world, n_cap):
    nbytes = lib.grinqh_allreduce_buffer_bytes(world, n_cap)
    p = ctypes.c_void_p()
    assert lib.grinqh_allreduce_buffer_alloc(nbytes, ctypes.byref(p)) == 0
    return p.value


@pytest.mark.parametrize("M", [1, 16])
def test_missing_rank_times_out_and_is_reported(monkeypatch, M):
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import grinqh.kernel  # noqa: F401
    from grinqh._ext import cabi
    from grinqh.utils import pack_codes
    lib = cabi()
    K, N, b = 2048, 4096, 8
    n_cap = M * N
    g = torch.Generator(device="cuda").manual_seed(3)
    w = pack_codes(torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g), b)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)

    def fused(world, bufs):
        if M == 1:
            return torch.ops.grinqh.gemv_allreduce(x, w, s, None, b, 128, N // 4, th, 0, world, bufs, n_cap)
        return torch.ops.grinqh.linear_allreduce(x, w, s, None, b, 128, N // 4, th, 0, 0, world, bufs, n_cap)

    th = [0.3, 0.6, 1.0, 1.5]
    own, silent = _alloc(lib, 2, n_cap), _alloc(lib, 2, n_cap)
    try:
        assert _take() == 0  # nothing pending from earlier tests
        monkeypatch.setenv("GRINQH_ALLREDUCE_WAIT_MS", "20")
        y = fused(2, [own, silent])
        torch.cuda.synchronize()  # the launch ends by itself
        assert _take() >= 1, "the wait for the missing rank was not reported"
        assert _take() == 0, "grinqh_take_error_flags did not clear the count"
        del y
        monkeypatch.delenv("GRINQH_ALLREDUCE_WAIT_MS")
        ref = fused(1, [own])
        plain = torch.ops.grinqh.gemm_or_gemv(x, w, s, None, b, 128, N // 4, th, False)
        if M == 1:
            assert torch.equal(ref, plain)
        else:  # the fused grid may split K differently (it must be resident at once)
            err = (ref.float() - plain.float()).abs().max() / plain.float().abs().max()
            assert err.item() <= 1e-2, f"max-rel {err.item():.3e} against the unfused GEMM"
        for _ in range(3):  # both buffer parities after the given-up launch
            assert torch.equal(fused(1, [own]), ref)
        assert _take() == 0
    finally:
        torch.cuda.synchronize()
        lib.grinqh_allreduce_buffer_free(ctypes.c_void_p(own))
        lib.grinqh_allreduce_buffer_free(ctypes.c_void_p(silent))
