"""The fused row-parallel kernel (torch.ops.grinqh.gemv_allreduce) with a single
rank: its peer-buffer path (epoch-tagged partials, bounded wait, ordered sum) must give exactly the
plain single-row GEMV's bits, over many consecutive launches (both buffer parities)
and under CUDA-graph replay. Runs on one GPU; the two-GPU test is
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
    p = PeerBuffers(None, n_cap=8192, device=torch.device("cuda", 0))
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
