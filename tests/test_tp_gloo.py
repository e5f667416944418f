"""Tensor-parallel composition on CPU with two gloo ranks: each rank loads its
shard through the plugin's weight loader, computes its partial output (the CPU
oracle stands in for the GPU kernel here; this test checks the sharding, not the
kernel), and the column / row-parallel collectives rebuild the TP=1 result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-grinqh-plugin_b200")]
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        import vllm.model_executor.parameter as P
        P.get_tensor_model_parallel_rank = lambda: rank
        P.get_tensor_model_parallel_world_size = lambda: world
        import oracle as O
        from grinqh import grinqh as G

        rng = np.random.default_rng(0)  # same data on every rank
        K, N, Gs, b = 256, 128, 128, 8
        codes = {name: rng.integers(-128, 128, size=(N, K)).astype(np.int8) for name in ("col", "row")}
        scl = {name: (rng.standard_normal((N, K // Gs)) * 0.01).astype(np.float32) for name in ("col", "row")}
        x = rng.standard_normal((3, K)).astype(np.float32)
        x = O.to_f32(O.round_to_dtype(x, "bf16"), "bf16")

        def layer_for(kl, parts, kfull):
            layer = torch.nn.Module()
            layer.tp_rank, layer.tp_size = rank, world
            m = G.GRINQHLinearMethod(G.GRINQHConfig(thresholds={}, max_bits=b), [0.0] * 4)
            m.create_weights(layer, kl, parts, kfull, N, torch.bfloat16)
            return layer

        def local_out(layer, name, xin):
            wp = layer.weight_packed
            wp.weight_loader(wp, torch.from_numpy(O.ct_pack_to_int32(codes[name], b)))
            layer.weight_scale.weight_loader(layer.weight_scale, torch.from_numpy(scl[name]).to(torch.bfloat16))
            c = wp.data.view(torch.int8).numpy()
            s = layer.weight_scale.data.float().numpy()
            return O.dense(xin, c, s, Gs, "bf16")  # fp64 partial (before the dtype cast)

        # column parallel: N split, outputs gathered
        yc = torch.from_numpy(local_out(layer_for(K, [N // world], K), "col", x))
        parts = [torch.empty_like(yc) for _ in range(world)]
        dist.all_gather(parts, yc)
        y_col = torch.cat(parts, dim=1).numpy()
        # row parallel: K split, partial outputs all-reduced
        kl = K // world
        yr = torch.from_numpy(local_out(layer_for(kl, [N], K), "row", x[:, rank * kl:(rank + 1) * kl]))
        dist.all_reduce(yr)
        y_row = yr.numpy()

        ref_col = O.dense(x, codes["col"].T, O.to_f32(O.round_to_dtype(scl["col"].T, "bf16"), "bf16"), Gs, "bf16")
        ref_row = O.dense(x, codes["row"].T, O.to_f32(O.round_to_dtype(scl["row"].T, "bf16"), "bf16"), Gs, "bf16")
        ok = np.allclose(y_col, ref_col, rtol=1e-12, atol=1e-9) and np.allclose(y_row, ref_row, rtol=1e-9, atol=1e-9)
        q.put((rank, bool(ok), ""))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        import traceback
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2])
def test_tp_column_and_row_parallel_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in results:
        assert ok, f"rank {rank}: {err}"
