"""Fused row-parallel linear on two GPUs: each rank runs the graded GEMV of its K slice
(torch.ops.grinqh.gemv_allreduce, one row) or the dense skinny GEMM of its K slice
(torch.ops.grinqh.linear_allreduce, 2..64 rows), and the same kernel sums the ranks'
partials over NVLink peer buffers. Checked against the CPU oracle of the unsharded
layer, for identical bits on both ranks, over many consecutive launches (the
device-side epoch and the double-buffered partials, shared by one-row and many-row
launches), under CUDA-graph replay, and timed against the unfused kernel followed by
an NCCL all-reduce. Needs two GPUs; skipped otherwise. NVLS is off
(NCCL_NVLS_ENABLE=0) and the kernels use plain peer stores only."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import FRO_TOL, MAX_REL_TOL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return (float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)),
            float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)))


def _worker(rank, world, port, q):
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-grinqh-plugin_b200")]
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        import oracle as O
        import grinqh.kernel  # noqa: F401
        from grinqh.allreduce import PeerBuffers, gemv_allreduce, linear_allreduce
        from grinqh.utils import pack_codes

        lines, ok = [], True
        rng = np.random.default_rng(0)  # same data on every rank

        def agree(flag):
            # every rank stops at the same point (after its kernels have finished), so no
            # rank exits while another may still write into its buffer
            torch.cuda.synchronize(dev)
            v = torch.tensor([1 if flag else 0], device=dev)
            dist.all_reduce(v, op=dist.ReduceOp.MIN)
            return bool(v.item())

        peers = PeerBuffers(None, n_cap=64 * 4096, device=dev)

        def bf16(a):
            return O.to_f32(O.round_to_dtype(np.asarray(a, np.float32), "bf16"), "bf16")

        def layer(K, N, b, G=128):
            codes = rng.integers(-(1 << (b - 1)), 1 << (b - 1), size=(K, N)).astype(np.int8)  # (K, N)
            scl = bf16(rng.random((K // G, N)) * 0.01 + 0.001)
            kl = K // world
            wr = pack_codes(torch.from_numpy(codes[rank * kl:(rank + 1) * kl]).to(dev), b)
            sr = torch.from_numpy(scl[rank * kl // G:(rank + 1) * kl // G]).to(dev).to(torch.bfloat16)
            return codes, scl, wr, sr, kl

        for (K, N, b, with_bias) in ((1024, 512, 8, False), (2048, 1024, 4, True), (4096, 4096, 8, False)):
            codes, scl, wr, sr, kl = layer(K, N, b)
            bias = bf16(rng.standard_normal(N) * 0.1) if with_bias else None
            bias_d = torch.from_numpy(bias).to(dev).to(torch.bfloat16) if with_bias else None
            cal = bf16(rng.standard_normal((64, K)))
            th = O.quantile_thresholds(np.abs(cal), [0.2, 0.4, 0.6, 0.8])
            worst = (0.0, 0.0)
            for it in range(12):  # consecutive launches: epochs and both buffer parities
                x = bf16(rng.standard_normal((1, K)))
                xd = torch.from_numpy(x[:, rank * kl:(rank + 1) * kl]).to(dev).to(torch.bfloat16)
                y = gemv_allreduce(xd, wr, sr, bias_d, b, 128, N // 4, th, peers)
                ys = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(ys, y)
                same = all(torch.equal(ys[0], t) for t in ys)
                ref = O.to_f32(O.gemm_or_gemv(x, codes, scl, bias, b, 128, th, "bf16"), "bf16")
                mx, fr = _rel(y.float().cpu().numpy(), ref)
                worst = (max(worst[0], mx), max(worst[1], fr))
                ok = ok and same and mx <= MAX_REL_TOL and fr <= FRO_TOL
                if not same:
                    lines.append(f"K={K} N={N} it={it}: ranks differ")
            lines.append(f"K={K} N={N} b={b} bias={with_bias}: worst max-rel {worst[0]:.2e} fro {worst[1]:.2e}")
            if not agree(ok):  # stop here on every rank: later phases would only repeat the failure
                raise RuntimeError("; ".join(lines))

        # 2..64 dense rows (batched decode): the skinny GEMM with the sum fused in,
        # single-row launches interleaved on the same buffers
        for (M, K, N, b, with_bias) in ((2, 1024, 512, 8, True), (16, 4096, 4096, 8, False),
                                        (64, 4096, 4096, 4, True), (64, 14336, 4096, 8, False)):
            codes, scl, wr, sr, kl = layer(K, N, b)
            bias = bf16(rng.standard_normal(N) * 0.1) if with_bias else None
            bias_d = torch.from_numpy(bias).to(dev).to(torch.bfloat16) if with_bias else None
            th = [0.3, 0.6, 1.0, 1.5]
            worst = (0.0, 0.0)
            for it in range(4):
                x = bf16(rng.standard_normal((M, K)))
                xd = torch.from_numpy(x[:, rank * kl:(rank + 1) * kl]).to(dev).to(torch.bfloat16).contiguous()
                y = linear_allreduce(xd, wr, sr, bias_d, b, 128, N // 4, th, peers)
                if it == 1:
                    gemv_allreduce(xd[:1], wr, sr, bias_d, b, 128, N // 4, th, peers)
                ys = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(ys, y)
                same = all(torch.equal(ys[0], t) for t in ys)
                ref = O.to_f32(O.gemm_or_gemv(x, codes, scl, bias, b, 128, th, "bf16"), "bf16")
                mx, fr = _rel(y.float().cpu().numpy(), ref)
                worst = (max(worst[0], mx), max(worst[1], fr))
                ok = ok and same and mx <= MAX_REL_TOL and fr <= FRO_TOL
                if not same:
                    lines.append(f"M={M} K={K} N={N} it={it}: ranks differ")
            lines.append(f"M={M} K={K} N={N} b={b} bias={with_bias}: worst max-rel {worst[0]:.2e} fro {worst[1]:.2e}")
            if not agree(ok):
                raise RuntimeError("; ".join(lines))

        # CUDA graph: three launches recorded, replayed with new inputs
        K, N, b = 2048, 2048, 8
        codes, scl, wr, sr, kl = layer(K, N, b)
        th = [0.3, 0.6, 1.0, 1.5]
        xs = [torch.zeros((1, kl), dtype=torch.bfloat16, device=dev) for _ in range(3)]
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for xx in xs:  # warm the per-stream workspace outside capture
                gemv_allreduce(xx, wr, sr, None, b, 128, N // 4, th, peers)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            outs = [gemv_allreduce(xx, wr, sr, None, b, 128, N // 4, th, peers) for xx in xs]
        for rep in range(4):
            xfull = [bf16(rng.standard_normal((1, K))) for _ in range(3)]
            for xx, xf in zip(xs, xfull):
                xx.copy_(torch.from_numpy(xf[:, rank * kl:(rank + 1) * kl]).to(torch.bfloat16))
            torch.cuda.synchronize(dev)
            dist.barrier()
            g.replay()
            torch.cuda.synchronize(dev)
            for o, xf in zip(outs, xfull):
                ref = O.to_f32(O.gemm_or_gemv(xf, codes, scl, None, b, 128, th, "bf16"), "bf16")
                mx, fr = _rel(o.float().cpu().numpy(), ref)
                ok = ok and mx <= MAX_REL_TOL and fr <= FRO_TOL
        lines.append(f"graph replays: last max-rel {mx:.2e} fro {fr:.2e}")
        del g
        if not agree(ok):
            raise RuntimeError("; ".join(lines))

        # timing: fused against the GEMV + NCCL all-reduce (o projection of Llama-3-8B at TP 2)
        K, N, b = 4096, 4096, 8
        codes, scl, wr, sr, kl = layer(K, N, b)
        xd = torch.from_numpy(bf16(rng.standard_normal((1, K)))[:, rank * kl:(rank + 1) * kl]).to(dev).to(torch.bfloat16)
        th = [0.3, 0.6, 1.0, 1.5]

        def fused():
            return gemv_allreduce(xd, wr, sr, None, b, 128, N // 4, th, peers)

        def unfused():
            y = torch.ops.grinqh.gemm_or_gemv(xd, wr, sr, None, b, 128, N // 4, th, False)
            dist.all_reduce(y)
            return y

        times = {}
        for name, fn in (("fused", fused), ("gemv+nccl", unfused)):
            for _ in range(20):
                fn()
            torch.cuda.synchronize(dev)
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(200):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            times[name] = e0.elapsed_time(e1) * 1e3 / 200
        # the same calls replayed from CUDA graphs (no host launch cost): the fused
        # kernel against the GEMV of the same slice alone, i.e. what the in-kernel sum adds
        def gemv_only():
            return torch.ops.grinqh.gemm_or_gemv(xd, wr, sr, None, b, 128, N // 4, th, False)

        st = torch.cuda.Stream(dev)
        for name, fn in (("fused graph", fused), ("gemv graph", gemv_only)):
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                fn()
            torch.cuda.current_stream(dev).wait_stream(st)
            torch.cuda.synchronize(dev)
            dist.barrier()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                for _ in range(50):
                    fn()
            torch.cuda.synchronize(dev)
            dist.barrier()
            gr.replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(4):
                gr.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            times[name] = e0.elapsed_time(e1) * 1e3 / 200
            del gr
        t = torch.tensor([times["fused"], times["gemv+nccl"], times["fused graph"], times["gemv graph"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        lines.append(f"K={K} N={N} TP={world}: eager fused {t[0].item():.1f} us, eager gemv + NCCL all-reduce "
                     f"{t[1].item():.1f} us; graph fused {t[2].item():.1f} us, graph gemv alone {t[3].item():.1f} us")
        # batch-64 decode at TP 2 (o and down of Llama-3-8B): the fused skinny GEMM
        # against the same GEMM followed by an NCCL all-reduce, both replayed from
        # CUDA graphs (the NCCL call captured in the graph) and eager
        for name, (K, N) in (("o", (4096, 4096)), ("down", (14336, 4096))):
            M, b = 64, 8
            codes, scl, wr, sr, kl = layer(K, N, b)
            xd = torch.from_numpy(bf16(rng.standard_normal((M, K)))[:, rank * kl:(rank + 1) * kl]).to(dev).to(
                torch.bfloat16).contiguous()
            th = [0.3, 0.6, 1.0, 1.5]

            def fused_rows():
                return linear_allreduce(xd, wr, sr, None, b, 128, N // 4, th, peers)

            def gemm_nccl():
                y = torch.ops.grinqh.gemm_or_gemv(xd, wr, sr, None, b, 128, N // 4, th, False)
                dist.all_reduce(y)
                return y

            rt = {}
            for tag, fn in (("fused", fused_rows), ("gemm+nccl", gemm_nccl)):
                for _ in range(10):
                    fn()
                torch.cuda.synchronize(dev)
                dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(100):
                    fn()
                e1.record()
                torch.cuda.synchronize(dev)
                rt[tag] = e0.elapsed_time(e1) * 1e3 / 100
                st = torch.cuda.Stream(dev)
                st.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(st):
                    fn()
                torch.cuda.current_stream(dev).wait_stream(st)
                torch.cuda.synchronize(dev)
                dist.barrier()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=st):
                    for _ in range(20):
                        fn()
                torch.cuda.synchronize(dev)
                dist.barrier()
                gr.replay()
                torch.cuda.synchronize(dev)
                dist.barrier()
                e0.record()
                for _ in range(5):
                    gr.replay()
                e1.record()
                torch.cuda.synchronize(dev)
                rt[tag + " graph"] = e0.elapsed_time(e1) * 1e3 / 100
                del gr
            t = torch.tensor([rt["fused"], rt["gemm+nccl"], rt["fused graph"], rt["gemm+nccl graph"]], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            lines.append(f"{name} M=64 K={K} N={N} TP={world}: eager fused {t[0].item():.1f} us vs GEMM + NCCL "
                         f"{t[1].item():.1f} us; graph fused {t[2].item():.1f} us vs GEMM + NCCL {t[3].item():.1f} us")

        from grinqh._ext import cabi
        import ctypes
        n_to = ctypes.c_uint(0)
        cabi().grinqh_take_error_flags(ctypes.byref(n_to))
        ok = ok and n_to.value == 0
        lines.append(f"wait timeouts {n_to.value}")
        peers.close()
        q.put((rank, bool(ok), "; ".join(lines)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report, never hang the parent
        import traceback
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_row_parallel_allreduce_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, msg in sorted(results):
        print(f"rank {rank}: {msg}")
    for rank, ok, msg in results:
        assert ok, f"rank {rank}: {msg}"
