"""Tensor parallelism on GPUs: two ranks over NCCL, each running the plugin's whole
path on its shard -- create_weights, the checkpoint loader narrowing by tensor-parallel
rank, process_weights_after_loading (pack on the GPU) and apply
(torch.ops.grinqh.gemm_or_gemv). Column-parallel outputs are all-gathered and
row-parallel partial outputs all-reduced, as vLLM does for these layers
(vllm/model_executor/layers/linear.py: ColumnParallelLinear gathers,
RowParallelLinear all-reduces); the result is compared with the CPU oracle of the
unsharded layer under the same composition (each rank's partial rounded to bf16, the
two partials summed and rounded once). Needs two GPUs; skipped otherwise."""
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


def _rel_errors(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    mx = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    fr = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    return float(mx), float(fr)


def _worker(rank, world, port, q):
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-grinqh-plugin_b200")]
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        import vllm.model_executor.parameter as P
        P.get_tensor_model_parallel_rank = lambda: rank
        P.get_tensor_model_parallel_world_size = lambda: world
        import oracle as O
        from grinqh import grinqh as G

        rng = np.random.default_rng(0)  # same data on every rank
        K, N, Gs, b = 1024, 512, 128, 8
        codes = {name: rng.integers(-128, 128, size=(N, K)).astype(np.int8) for name in ("col", "row")}
        scl = {name: O.to_f32(O.round_to_dtype((rng.random((N, K // Gs)) * 0.01 + 0.001).astype(np.float32),
                                                "bf16"), "bf16") for name in ("col", "row")}
        cal = O.to_f32(O.round_to_dtype(rng.standard_normal((64, K)).astype(np.float32), "bf16"), "bf16")
        th = O.quantile_thresholds(np.abs(cal), [0.2, 0.4, 0.6, 0.8])

        def layer_for(kl, parts, name):
            with torch.device(dev):
                layer = torch.nn.Module()
                layer.tp_rank, layer.tp_size = rank, world
                m = G.GRINQHLinearMethod(G.GRINQHConfig(thresholds={}, max_bits=b), th)
                m.create_weights(layer, kl, parts, K, N, torch.bfloat16)
            wp = layer.weight_packed
            wp.weight_loader(wp, torch.from_numpy(O.ct_pack_to_int32(codes[name], b)))
            layer.weight_scale.weight_loader(layer.weight_scale, torch.from_numpy(scl[name]).to(torch.bfloat16))
            m.process_weights_after_loading(layer)
            return layer, m

        lines = []
        ok = True
        col, mcol = layer_for(K, [N // world], "col")
        kl = K // world
        row, mrow = layer_for(kl, [N], "row")
        for M in (1, 16):
            x = O.to_f32(O.round_to_dtype(rng.standard_normal((M, K)).astype(np.float32), "bf16"), "bf16")
            xd = torch.from_numpy(x).to(dev).to(torch.bfloat16)

            # column parallel: this rank's N slice, gathered along N
            yc = mcol.apply(col, xd)
            parts = [torch.empty_like(yc) for _ in range(world)]
            dist.all_gather(parts, yc)
            y_col = torch.cat(parts, dim=1).float().cpu().numpy()
            ref_col = O.gemm_or_gemv(x, codes["col"].T, scl["col"].T, None, b, Gs, th, "bf16")

            # row parallel: this rank's K slice, partial outputs all-reduced
            yr = mrow.apply(row, xd[:, rank * kl:(rank + 1) * kl].contiguous())
            dist.all_reduce(yr)
            y_row = yr.float().cpu().numpy()
            partials = [O.to_f32(O.gemm_or_gemv(x[:, r * kl:(r + 1) * kl], codes["row"].T[r * kl:(r + 1) * kl],
                                                scl["row"].T[r * kl // Gs:(r + 1) * kl // Gs], None, b, Gs, th,
                                                "bf16"), "bf16") for r in range(world)]
            ref_row = O.to_f32(O.round_to_dtype(sum(p.astype(np.float64) for p in partials).astype(np.float32),
                                                "bf16"), "bf16")
            for tag, got, ref in (("column", y_col, O.to_f32(ref_col, "bf16")), ("row", y_row, ref_row)):
                mx, fr = _rel_errors(got, ref)
                good = mx <= MAX_REL_TOL and fr <= FRO_TOL
                ok = ok and good
                lines.append(f"M={M} {tag}: max-rel {mx:.2e} fro {fr:.2e}")
        q.put((rank, bool(ok), "; ".join(lines)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report, never hang the parent
        import traceback
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_column_and_row_parallel_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, msg in results:
        assert ok, f"rank {rank}: {msg}"
