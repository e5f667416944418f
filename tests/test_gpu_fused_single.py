"""The fused row-parallel kernels with a single rank: the single-row GEMV
(torch.ops.grinqh.gemv_allreduce) through its peer-buffer path (epoch-tagged partials,
bounded wait, ordered sum) must give exactly the plain single-row GEMV's bits, over
many consecutive launches (both buffer parities) and under CUDA-graph replay; the
skinny dense GEMM of 2..64 rows (torch.ops.grinqh.linear_allreduce) must match the
CPU oracle of the dense path and be deterministic, also when single-row and
multi-row launches share the buffers' epochs. Runs on one GPU; the two-GPU test is
test_tp_fused_allreduce.py."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def peers():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import grinqh.kernel  # noqa: F401
    from grinqh.allreduce import PeerBuffers
    own_group = not dist.is_initialized()
    if own_group:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    p = PeerBuffers(None, n_cap=64 * 8192, device=torch.device("cuda", 0))
    yield p
    p.close()
    if own_group:
        dist.destroy_process_group()


@pytest.mark.parametrize("b,K,N,bias", [(8, 1024, 512, False), (4, 4096, 4096, True), (2, 2048, 8192, False),
                                        (6, 512, 1056, True)])
def test_single_rank_matches_plain_gemv(peers, b, K, N, bias):
    from grinqh.allreduce import gemv_allreduce
    from grinqh.utils import pack_codes
    g = torch.Generator(device="cuda").manual_seed(b * 7 + K)
    codes = torch.randint(-(1 << (b - 1)), 1 << (b - 1), (K, N), dtype=torch.int8, device="cuda", generator=g)
    w = pack_codes(codes, b)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    bv = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16) if bias else None
    th = [0.3, 0.6, 1.0, 1.5]
    for it in range(9):  # both parities, several epochs
        x = torch.randn(1, K, device="cuda", generator=g).to(torch.bfloat16)
        y = gemv_allreduce(x, w, s, bv, b, 128, N // 4, th, peers)
        ref = torch.ops.grinqh.gemm_or_gemv(x, w, s, bv, b, 128, N // 4, th, False)
        assert torch.equal(y, ref), f"launch {it}: max diff {(y.float() - ref.float()).abs().max().item()}"


def test_single_rank_graph_replay(peers):
    from grinqh.allreduce import gemv_allreduce
    from grinqh.utils import pack_codes
    K, N, b = 2048, 2048, 8
    g = torch.Generator(device="cuda").manual_seed(5)
    w = pack_codes(torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g), b)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    th = [0.3, 0.6, 1.0, 1.5]
    xs = [torch.zeros(1, K, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for xx in xs:
            gemv_allreduce(xx, w, s, None, b, 128, N // 4, th, peers)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        outs = [gemv_allreduce(xx, w, s, None, b, 128, N // 4, th, peers) for xx in xs]
    for rep in range(5):
        for xx in xs:
            xx.copy_(torch.randn(1, K, device="cuda", generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        for xx, o in zip(xs, outs):
            ref = torch.ops.grinqh.gemm_or_gemv(xx, w, s, None, b, 128, N // 4, th, False)
            assert torch.equal(o, ref), f"replay {rep}"
    import ctypes
    from grinqh._ext import cabi
    n = ctypes.c_uint(0)
    cabi().grinqh_take_error_flags(ctypes.byref(n))
    assert n.value == 0


@pytest.mark.parametrize("M,K,N,b,bias,dt", [(2, 1024, 512, 8, False, "bf16"), (16, 7168, 4096, 8, True, "bf16"),
                                             (64, 2048, 4096, 4, False, "f16"), (40, 512, 1088, 2, True, "bf16"),
                                             (5, 4096, 14336, 6, False, "f16")])
def test_single_rank_rows_match_oracle(peers, M, K, N, b, bias, dt):
    import oracle as O
    from conftest import FRO_TOL, MAX_REL_TOL, rel_errors
    from grinqh.allreduce import gemv_allreduce, linear_allreduce
    from grinqh.utils import pack_codes
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    g = torch.Generator(device="cuda").manual_seed(M * 131 + K + b)
    codes = torch.randint(-(1 << (b - 1)), 1 << (b - 1), (K, N), dtype=torch.int8, device="cuda", generator=g)
    w = pack_codes(codes, b)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(tdt)
    bv = (torch.randn(N, device="cuda", generator=g) * 0.1).to(tdt) if bias else None
    th = [0.3, 0.6, 1.0, 1.5]
    codes_np, s_np = codes.cpu().numpy(), s.float().cpu().numpy()
    b_np = bv.float().cpu().numpy() if bias else None
    x1 = torch.randn(1, K, device="cuda", generator=g).to(tdt)
    for it in range(5):  # both parities; single-row launches interleaved on the same epochs
        x = torch.randn(M, K, device="cuda", generator=g).to(tdt)
        y = linear_allreduce(x, w, s, bv, b, 128, N // 4, th, peers)
        y2 = linear_allreduce(x, w, s, bv, b, 128, N // 4, th, peers)
        assert torch.equal(y, y2), f"launch {it}: not deterministic"
        if it % 2 == 0:
            y1 = gemv_allreduce(x1, w, s, bv, b, 128, N // 4, th, peers)
            assert torch.equal(y1, torch.ops.grinqh.gemm_or_gemv(x1, w, s, bv, b, 128, N // 4, th, False))
        ref = O.gemm_or_gemv(x.float().cpu().numpy(), codes_np, s_np, b_np, b, 128, th, dt)
        mx, fr = rel_errors(y.float().cpu().numpy(), O.to_f32(ref, dt))
        assert mx <= MAX_REL_TOL and fr <= FRO_TOL, f"launch {it}: max-rel {mx:.3e}, fro {fr:.3e}"
    import ctypes
    from grinqh._ext import cabi
    n = ctypes.c_uint(0)
    cabi().grinqh_take_error_flags(ctypes.byref(n))
    assert n.value == 0


def test_single_rank_rows_graph_replay(peers):
    from grinqh.allreduce import linear_allreduce
    from grinqh.utils import pack_codes
    M, K, N, b = 32, 2048, 4096, 8
    g = torch.Generator(device="cuda").manual_seed(9)
    w = pack_codes(torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g), b)
    s = (torch.rand(K // 128, N, device="cuda", generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    th = [0.3, 0.6, 1.0, 1.5]
    xs = [torch.zeros(M, K, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for xx in xs:
            linear_allreduce(xx, w, s, None, b, 128, N // 4, th, peers)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        outs = [linear_allreduce(xx, w, s, None, b, 128, N // 4, th, peers) for xx in xs]
    for rep in range(4):
        for xx in xs:
            xx.copy_(torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        for xx, o in zip(xs, outs):
            ref = linear_allreduce(xx, w, s, None, b, 128, N // 4, th, peers)  # eager, same plan
            assert torch.equal(o, ref), f"replay {rep}"


def test_fused_refuses_unsupported_rows(peers):
    """Shapes outside the fused kernels are refused before launch with the message the
    plugin's fallback looks for: graded rows beyond one, dense rows beyond 64."""
    from grinqh.allreduce import linear_allreduce
    from grinqh.utils import pack_codes
    K, N, b = 512, 512, 8
    w = pack_codes(torch.zeros((K, N), dtype=torch.int8, device="cuda"), b)
    s = torch.ones(K // 128, N, dtype=torch.bfloat16, device="cuda")
    th = [0.3, 0.6, 1.0, 1.5]
    for M, mode in ((65, 0), (4, 2)):
        with pytest.raises(RuntimeError, match="fused all-reduce not supported"):
            linear_allreduce(torch.zeros(M, K, dtype=torch.bfloat16, device="cuda"), w, s, None, b, 128, N // 4, th,
                             peers, mode=mode)
