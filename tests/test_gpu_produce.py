"""Producers of x with the grading fused in (csrc/produce.cu): vLLM's RMSNorm (with and
without the residual add) and SiLU(gate) * up, each writing the next linear's input,
its grade masks and their union over the rows; and the batch-union GEMV fed with that
union. Checked against torch on the same GPU for the produced values (vLLM's own
formulas, vllm/ir/ops/layernorm.py:10-58 and SiluAndMul.forward_native: at most one
unit in the last place apart, from the order of the fp32 sum of squares), bit-exact for
the residual, and bit-exact against the CPU oracle's grade (grinqh/kernel.py:100-116)
of the produced values for the masks and the union."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import grinqh.kernel  # noqa: F401


def _ulps(a, b):
    """Distance in units in the last place between two bf16 / fp16 tensors (same sign
    assumed where both are non-zero; sign changes count as large)."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    # sign-magnitude -> ordered integers
    oa = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ob = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return (oa - ob).abs()


def _check_grades(out, masks, uni, th, bits):
    o32 = out.float().cpu().numpy().reshape(-1, out.shape[-1])
    want = O.grade(o32, th, bits)
    got = masks.cpu().numpy().reshape(want.shape)
    assert np.array_equal(got, want), f"{int((got != want).sum())} mask bytes differ"
    assert np.array_equal(uni.cpu().numpy(), np.bitwise_or.reduce(want, axis=0)), "union differs"


def _rms_ref(x, residual, weight, eps):
    """vllm/ir/ops/layernorm.py:10-58 in torch (fp32 on the GPU)."""
    xf = x.float()
    new_res = None
    if residual is not None:
        xf = xf + residual.float()
        new_res = xf.to(x.dtype)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps)
    if weight is not None:
        y = y.to(weight.dtype) * weight
    return y.to(x.dtype), new_res


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,bits,with_res,with_w", [(1, 4096, 8, False, True), (7, 4096, 4, True, True),
                                                      (64, 8192, 6, True, True), (3, 1032, 2, False, False),
                                                      (33, 14336, 8, True, True)])
def test_rmsnorm_grade(dt, M, K, bits, with_res, with_w):
    from grinqh.kernel import grinqh_rmsnorm_grade
    g = torch.Generator(device="cuda").manual_seed(M * 7 + K + bits)
    x = (torch.randn(M, K, device="cuda", generator=g) * 3).to(dt)
    res = (torch.randn(M, K, device="cuda", generator=g) * 2).to(dt) if with_res else None
    w = (torch.rand(K, device="cuda", generator=g) + 0.5).to(dt) if with_w else None
    ref, ref_res = _rms_ref(x, res, w, 1e-6)
    res_in = res.clone() if with_res else None
    th = [0.4, 0.8, 1.3, 2.0]
    out, masks, uni = grinqh_rmsnorm_grade(x, res_in, w, 1e-6, th, bits)
    d = _ulps(out, ref)
    assert int(d.max()) <= 1, f"max {int(d.max())} ulp"
    assert float((d > 0).float().mean()) < 0.02, "too many outputs off by one ulp"
    if with_res:
        assert torch.equal(res_in, ref_res), "residual differs from dtype(x + residual)"
    _check_grades(out, masks, uni, th, bits)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,bits", [(1, 14336, 8), (16, 14336, 4), (5, 1000, 6), (64, 2048, 2)])
def test_silu_mul_grade(dt, M, K, bits):
    from grinqh.kernel import grinqh_silu_mul_grade
    g = torch.Generator(device="cuda").manual_seed(M + K + bits)
    x = (torch.randn(M, 2 * K, device="cuda", generator=g) * 2).to(dt)
    ref = F.silu(x[:, :K]) * x[:, K:]
    th = [0.05, 0.2, 0.6, 1.5]
    out, masks, uni = grinqh_silu_mul_grade(x, th, bits)
    d = _ulps(out, ref)
    assert int(d.max()) <= 1, f"max {int(d.max())} ulp"
    _check_grades(out, masks, uni, th, bits)


def test_producer_edge_cases():
    from grinqh.kernel import grinqh_rmsnorm_grade, grinqh_silu_mul_grade
    th = [0.1, 0.2, 0.3, 0.4]
    out, masks, uni = grinqh_rmsnorm_grade(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda"), None, None,
                                           1e-5, th, 8)
    assert out.shape == (0, 256) and torch.equal(uni, torch.zeros(256, dtype=torch.uint8, device="cuda"))
    # a zero row: rsqrt(eps) * 0 = 0, graded 0 everywhere
    out, masks, uni = grinqh_rmsnorm_grade(torch.zeros(2, 512, dtype=torch.bfloat16, device="cuda"), None, None,
                                           1e-5, th, 8)
    assert int(out.float().abs().max()) == 0 and int(masks.max()) == 0 and int(uni.max()) == 0
    with pytest.raises(RuntimeError, match="multiple of 8"):
        grinqh_silu_mul_grade(torch.zeros(2, 12, dtype=torch.bfloat16, device="cuda"), th, 8)


@pytest.mark.parametrize("M,K,N,bits", [(4, 4096, 4096, 8), (16, 14336, 1024, 4), (2, 1024, 512, 6)])
def test_union_gemv_with_producer_union(M, K, N, bits):
    """The batch-union GEMV fed with the producer's union gives the bits of the GEMV
    that grades its rows itself, and both match the CPU oracle."""
    from grinqh.kernel import (grinqh_gemv_batch_union, grinqh_gemv_batch_union_masked, grinqh_rmsnorm_grade,
                               grinqh_silu_mul_grade)
    from grinqh.utils import pack_codes
    g = torch.Generator(device="cuda").manual_seed(K + N + M)
    codes = torch.randint(-(1 << (bits - 1)), 1 << (bits - 1), (K, N), dtype=torch.int8, device="cuda", generator=g)
    w = pack_codes(codes, bits)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    th = [0.3, 0.7, 1.2, 2.0]
    h = torch.randn(M, 2 * K, device="cuda", generator=g).to(torch.bfloat16)
    for producer in ("rmsnorm", "silu_mul"):
        if producer == "rmsnorm":
            x, _, uni = grinqh_rmsnorm_grade(h[:, :K].contiguous(), None, None, 1e-6, th, bits)
        else:
            x, _, uni = grinqh_silu_mul_grade(h, th, bits)
        y_self = grinqh_gemv_batch_union(x, w, s, None, bits, 128, N // 4, th)
        y_fed = grinqh_gemv_batch_union_masked(x, w, s, None, bits, 128, N // 4, th, uni)
        assert torch.equal(y_self, y_fed), f"{producer}: the fed union changes the result"
        xs = x.float().cpu().numpy()
        ref = O.to_f32(O.round_to_dtype(O.union_gemv(xs, codes.cpu().numpy(), s.float().cpu().numpy(), th, bits,
                                                     128), "bf16"), "bf16")
        got = y_fed.float().cpu().numpy()
        mx = float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert mx <= 1e-2, f"{producer}: max-rel {mx:.3e} against the oracle"
