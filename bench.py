#!/usr/bin/env python
"""GRINQH quantized-linear benchmark (B200, sm_100a).

Workload (configs[1] of the baseline, Llama-3-8B linear shapes): one decoder
layer's four quantized linears -- qkv 4096->6144, o 4096->4096, gate_up
4096->28672, down 14336->4096 -- b = 8 bit weights in bit planes, group 128, bf16
activations. A *step* is one pass of the hot path over one batch: the four linears
at the decode batch M (default 1: the graded GEMV, thresholds = quantiles
.2/.4/.6/.8 of a 512-token calibration batch).

Metric: algorithmic HBM bytes / second over the whole job (weight planes the
grades select + scales of touched groups + activations + outputs). Two copies of
the layer's weights are rotated (436 MB at b=8 > 126 MB L2), so every step reads
its weights from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun). By default the ranks run the layer
tensor-parallel as vLLM shards it (qkv / gate_up column parallel, o / down row
parallel with the partial sums added in the step: the fused GEMV + all-reduce kernel
for one row, NCCL otherwise) -- strong scaling, the value is the layer's bytes over
the max-over-ranks time, and every run checks the sharded outputs against the
unsharded layer. `--replicas` runs the single-GPU workload on every rank instead
(weak scaling, no collective on the data path).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-grinqh-plugin_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

SHAPES = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 28672), "down": (14336, 4096)}
GROUP = 128
QUANTILES = [0.2, 0.4, 0.6, 0.8]
FUSED_MAX_ROWS = 64  # rows the fused row-parallel kernels take (grinqh.allreduce.FUSED_MAX_ROWS)


PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "m1_kernel_gate_up_b8_graded.md")


def _committed_traffic(kernel_tag):
    """DRAM bytes (read + write) of one launch of the dominant kernel, from the
    committed ncu summary of this benchmark's own launch (a line
    `traffic_bytes_per_launch: <bytes>` next to `kernel_tag: <tag>`), else None."""
    try:
        with open(PROFILE_SUMMARY) as f:
            kv = dict(l.strip().split(": ", 1) for l in f if l.startswith(("traffic_bytes_per_launch:", "kernel_tag:")))
        if kv.get("kernel_tag") == kernel_tag:
            return int(kv["traffic_bytes_per_launch"])
    except Exception:
        pass
    return None


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ----------------------------------------------------------------------------- data
ROW_PARALLEL = ("o", "down")  # vLLM RowParallelLinear (K sharded, partial sums all-reduced)


def make_codes(dev, bits, seed, name):
    """RTN-quantized N(0, 0.02) weights of one linear: int8 codes (K, N), bf16 scales."""
    K, N = SHAPES[name]
    g = torch.Generator(device=dev).manual_seed(seed * 16 + list(SHAPES).index(name))
    qmax = (1 << (bits - 1)) - 1
    w = torch.randn((K, N), generator=g, device=dev) * 0.02
    s = (w.view(K // GROUP, GROUP, N).abs().amax(1) / qmax).clamp_min(1e-8).to(torch.bfloat16)
    codes = torch.clamp(torch.round(w / s.float().repeat_interleave(GROUP, 0)), -qmax - 1, qmax).to(torch.int8)
    return codes, s


def shard(codes, s, name, rank, world):
    """This rank's tensor-parallel shard: o / down keep a K slice (row parallel), qkv /
    gate_up an N slice (column parallel; one contiguous slice of the merged output,
    which moves the same bytes as vLLM's per-sub-matrix slices)."""
    K, N = SHAPES[name]
    if name in ROW_PARALLEL:
        kl = K // world
        return codes[rank * kl:(rank + 1) * kl], s[rank * kl // GROUP:(rank + 1) * kl // GROUP]
    nl = N // world
    return codes[:, rank * nl:(rank + 1) * nl], s[:, rank * nl:(rank + 1) * nl]


def make_layer(dev, bits, seed, rank=0, world=1):
    """The layer's four linears as bit planes (this rank's shards when world > 1)."""
    from grinqh.utils import pack_codes
    layer = {}
    for name in SHAPES:
        codes, s = make_codes(dev, bits, seed, name)
        if world > 1:
            codes, s = shard(codes, s, name, rank, world)
        layer[name] = (pack_codes(codes.contiguous(), bits), s.contiguous())
        del codes
    return layer


def layer_bytes(layer):
    return sum(w.numel() * 4 + s.numel() * 2 for w, s in layer.values())


class StepGraphs:
    """CUDA graphs that replay `step(copy)` over rotating weight copies, so that K timed
    steps run K captured steps and nothing eagerly: `ncopies` graphs of G steps (graph c
    runs copies (c G + t) mod ncopies, so consecutive replays continue the rotation) and
    one graph for the remainder K mod G."""

    def __init__(self, step, ncopies, steps, stream, G=8):
        self.G, self.nc = G, ncopies
        self.full, rem = divmod(steps, G)
        self.graphs = []
        with torch.cuda.stream(stream):
            for c in range(ncopies):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for t in range(G):
                        step((c * G + t) % ncopies)
                self.graphs.append(g)
            self.rem = None
            if rem:
                start = (self.full * G) % ncopies
                self.rem = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.rem, stream=stream):
                    for t in range(rem):
                        step((start + t) % ncopies)

    def replay(self, nfull=None):
        for i in range(self.full if nfull is None else nfull):
            self.graphs[i % self.nc].replay()
        if nfull is None and self.rem is not None:
            self.rem.replay()


def make_inputs(dev, M, seed):
    """bf16 N(0,1) activations, 1% fixed outlier channels x20; thresholds from a
    seeded 512-token calibration batch of the same distribution."""
    g = torch.Generator(device=dev).manual_seed(seed)
    xs, ths = {}, {}
    for name, (K, N) in SHAPES.items():
        idx = torch.randperm(K, generator=g, device=dev)[: max(1, K // 100)]
        x = torch.randn((M, K), generator=g, device=dev)
        x[:, idx] *= 20
        cal = torch.randn((512, K), generator=g, device=dev)
        cal[:, idx] *= 20
        a = cal.to(torch.bfloat16).abs().float().flatten()
        # torch.quantile is limited to 16M elements: sort-based linear interpolation
        srt = torch.sort(a).values
        th = []
        for q in QUANTILES:
            pos = q * (srt.numel() - 1)
            lo = int(math.floor(pos))
            hi = min(lo + 1, srt.numel() - 1)
            th.append(float(srt[lo] + (srt[hi] - srt[lo]) * (pos - lo)))
        xs[name] = x.to(torch.bfloat16)
        ths[name] = th
    return xs, ths


def algorithmic_bytes(xs, ths, bits, M, graded, shapes=None):
    """Bytes one step must move: active planes (union over rows) + touched scale
    groups + x + y, per linear (roofline definition of the hot path). `shapes`: the
    (K, N) each linear has on this GPU (its tensor-parallel shard), `xs` its inputs."""
    from grinqh.kernel import grinqh_grade
    per = {}
    for name, (K, N) in (shapes or SHAPES).items():
        if graded:
            _, uni = grinqh_grade(xs[name], ths[name], bits)
            u = uni.to(torch.int32)
            planes = int(sum(((u >> z) & 1).sum().item() for z in range(bits // 2)))
            groups = int((uni.view(K // GROUP, GROUP) != 0).any(1).sum().item())
        else:
            planes, groups = K * (bits // 2), K // GROUP
        per[name] = planes * (N // 4) + groups * N * 2 + 2 * M * K + 2 * M * N
    return per


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """NVML sampling of SM clock and throttle reasons (read-only queries)."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap", 0x1: "gpu_idle"}

    def __init__(self, index):
        self.samples, self.ok = [], False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                try:
                    rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    rs = self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self, t0, t1):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-3:]
        reasons = set()
        for _, _, rs in inside:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(inside)}


# ----------------------------------------------------------------------------- ours
def run_ours(args, rank, world, dev):
    """The timed step on this rank. One GPU (or --replicas): the layer's four linears,
    two weight copies rotated. Several GPUs (default): tensor parallelism as vLLM
    shards the layer -- qkv and gate_up column parallel, o and down row parallel with
    the ranks' partial sums added in the step (the fused GEMV + all-reduce kernel for
    one row, the fused skinny GEMM + all-reduce kernel for 2..64 rows, the GEMM followed
    by NCCL's all-reduce for more rows)."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    bits, M = args.bits, args.m
    torch.cuda.set_device(dev)
    tp = world > 1 and not args.replicas
    graded = M == 1
    if tp:
        probe = make_layer(dev, bits, 0, rank, world)
        ncopies = max(2, math.ceil(2 * L2_BYTES / layer_bytes(probe)))
        layers = [probe] + [make_layer(dev, bits, c, rank, world) for c in range(1, ncopies)]
        xs, ths = make_inputs(dev, M, 7)  # the same activations on every rank
    else:
        ncopies = 2  # 2 x 222 MB > L2
        layers = [make_layer(dev, bits, 1000 * rank + c) for c in range(ncopies)]
        xs, ths = make_inputs(dev, M, 7 + rank)
    local = {}  # this rank's (K, N) per linear
    x_in = {}   # activations each linear reads (row-parallel: the rank's K slice)
    for name, (K, N) in SHAPES.items():
        if tp and name in ROW_PARALLEL:
            kl = K // world
            local[name] = (kl, N)
            x_in[name] = xs[name][:, rank * kl:(rank + 1) * kl].contiguous()
        else:
            local[name] = (K, N // world if tp else N)
            x_in[name] = xs[name]
    per = algorithmic_bytes(x_in, ths, bits, M, graded, local)
    step_bytes = sum(per.values())
    if world > 1:
        t = torch.tensor([step_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        job_step_bytes = float(t.item())
    else:
        job_step_bytes = float(step_bytes)

    peers = None
    ctrl = None
    if tp:
        ctrl = dist.new_group(backend="gloo")
        if M <= FUSED_MAX_ROWS:
            from grinqh.allreduce import PeerBuffers
            peers = PeerBuffers(ctrl, n_cap=M * max(SHAPES[n][1] for n in ROW_PARALLEL), device=dev)

    def run_linear(c, name, fused=True):
        w, s = layers[c][name]
        kl, nl = local[name]
        if tp and name in ROW_PARALLEL and fused:
            if graded:
                from grinqh.allreduce import gemv_allreduce
                return gemv_allreduce(x_in[name], w, s, None, bits, GROUP, nl // 4, ths[name], peers)
            if M <= FUSED_MAX_ROWS:
                from grinqh.allreduce import linear_allreduce
                return linear_allreduce(x_in[name], w, s, None, bits, GROUP, nl // 4, ths[name], peers)
            y = grinqh_gemm_or_gemv(x_in[name], w, s, None, bits, GROUP, nl // 4, ths[name])
            dist.all_reduce(y)
            return y
        return grinqh_gemm_or_gemv(x_in[name], w, s, None, bits, GROUP, nl // 4, ths[name])

    def step(c, fused=True):
        return [run_linear(c, name, fused) for name in SHAPES]

    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):  # warm the allocator / lazy init before capture
            step(0)
    torch.cuda.synchronize(dev)

    tp_check = None
    if tp:
        tp_check = check_tp_outputs(dev, bits, M, xs, ths, x_in, local, layers[0], step, rank, world, stream)

    graphs = StepGraphs(step, ncopies, args.steps, stream)
    warm = StepGraphs(step, ncopies, max(args.warmup, 3), stream)
    with torch.cuda.stream(stream):
        warm.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(dev.index if dev.index is not None else 0).start()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_host0 = time.perf_counter()
    with torch.cuda.stream(stream):
        e0.record(stream)
        graphs.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    t_host1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1), dev, world)
    value = job_step_bytes * args.steps / (ms / 1e3) / 1e9

    allreduce_us = None
    if tp:
        # the same step with the row-parallel linears' sums left out: the difference is
        # what the tensor-parallel sum costs per step (max over ranks of both)
        plain = StepGraphs(lambda c: step(c, fused=False), ncopies, args.steps, stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            plain.replay(2)
            p0.record(stream)
            plain.replay()
            p1.record(stream)
        torch.cuda.synchronize(dev)
        ms_plain = max_over_ranks(p0.elapsed_time(p1), dev, world)
        allreduce_us = (ms - ms_plain) * 1e3 / args.steps
        del plain

    # ---- dominant kernel (gate_up) alone: average launch duration over rotating copies
    name = "gate_up"
    K, N = local[name]
    R = 64
    with torch.cuda.stream(stream):
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gk, stream=stream):
            for i in range(R):
                w, s = layers[i % ncopies][name]
                grinqh_gemm_or_gemv(x_in[name], w, s, None, bits, GROUP, N // 4, ths[name])
        gk.replay()
        torch.cuda.synchronize(dev)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(5):
            gk.replay()
        k1.record(stream)
    torch.cuda.synchronize(dev)
    kern_ms = k0.elapsed_time(k1) / (5 * R)
    hbm_peak, tc_peak, peak_src = _peaks()
    achieved = per[name] / (kern_ms / 1e3) / 1e9

    e2e_ms, h2d, d2h = run_e2e(args, dev, stream, layers, ncopies, x_in, xs, ths, local, peers, tp, rank, world)
    e2e_value = job_step_bytes / (e2e_ms / 1e3) / 1e9

    sweep = None if (args.no_sweep or world > 1) else m_sweep(layers, bits, dev, stream)
    skew = None if (args.no_sweep or world > 1) else grade_skew(bits, dev, stream)

    if tp:
        parallelism = (f"tp{world}: qkv / gate_up column parallel, o / down row parallel with the sum "
                       + ("fused into the GEMV (NVLink peer stores)" if graded else
                          "fused into the skinny GEMM (NVLink peer stores)" if M <= FUSED_MAX_ROWS
                          else "by NCCL all-reduce"))
    else:
        parallelism = f"replicas x{world} (no collective on the data path)"
    line = {
        "metric": "quant-linear HBM GB/s, Llama-3-8B layer linears (qkv+o+gate_up+down), decode",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 6), "higher_is_better": True,
        "scaling": "strong" if tp else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"configs[1] Llama-3-8B linear shapes, M={M} "
                               f"{'graded GEMV (quantile .2/.4/.6/.8 thresholds)' if graded else 'dense'}, "
                               f"b={bits}, group {GROUP}",
                   "shapes": {k: list(v) for k, v in SHAPES.items()}, "M": M, "max_bits": bits,
                   "group_size": GROUP, "algorithmic_bytes_per_step": job_step_bytes,
                   "l2": "inputs larger than L2: %d weight copies rotated (%.0f MB per copy per GPU)" %
                         (ncopies, layer_bytes(layers[0]) / 1e6),
                   "parallelism": parallelism,
                   "timing": "CUDA events around CUDA-graph replays of the K steps (every step captured)"},
        "roofline": {"bound": "hbm", "kernel": f"{name} graded GEMV" if graded else f"{name} dense",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
                     "bytes_per_launch": per[name], "avg_launch_us": round(kern_ms * 1e3, 3),
                     "traffic": _committed_traffic(f"m1_kernel gate_up b{bits} M{M} graded") if graded and not tp
                     else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the bench's own gate_up "
                                       "launch, profiles/m1_kernel_gate_up_b8_graded.md"},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks.summary(t_host0, t_host1),
        "per_linear_bytes": per,
    }
    if tp:
        line["tp_check"] = tp_check
        line["allreduce_us_per_step"] = round(allreduce_us, 3)
        line["allreduce_share"] = round(allreduce_us * 1e-3 * args.steps / ms, 4)
    if sweep is not None:
        line["m_sweep"] = sweep
    if skew is not None:
        line["grade_skew"] = skew
    if peers is not None:
        del graphs, warm
        peers.close()
    return line


L2_BYTES = 126e6


def max_over_ranks(ms, dev, world):
    if world == 1:
        return ms
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_tp_outputs(dev, bits, M, xs, ths, x_in, local, shards, step, rank, world, stream):
    """Every rank's outputs of one sharded step against the same layer unsharded on
    this GPU (the single-GPU path, itself checked against the CPU oracle by the GPU
    tests): column-parallel shards against their columns of the full output, the
    summed row-parallel outputs against the full output. Max over ranks of the
    max-normalised and relative-Frobenius errors; the bar is the parity bar."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    worst = [0.0, 0.0]
    with torch.cuda.stream(stream):
        outs = step(0)
        for out, (name, (K, N)) in zip(outs, SHAPES.items()):
            codes, s = make_codes(dev, bits, 0, name)
            full = grinqh_gemm_or_gemv(xs[name], pack_codes(codes, bits), s, None, bits, GROUP, N // 4, ths[name])
            if name not in ROW_PARALLEL:
                nl = local[name][1]
                full = full[:, rank * nl:(rank + 1) * nl]
            d = (out.float() - full.float())
            mx = (d.abs().max() / full.float().abs().max().clamp_min(1e-30)).item()
            fro = (d.norm() / full.float().norm().clamp_min(1e-30)).item()
            worst = [max(worst[0], mx), max(worst[1], fro)]
            del codes, full
    torch.cuda.synchronize(dev)
    t = torch.tensor(worst, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    mx, fro = t.tolist()
    return {"max_rel": mx, "fro": fro, "pass": bool(mx <= 1e-2 and fro <= 2e-3),
            "against": "the unsharded layer on one GPU, every linear, max over ranks"}


def run_e2e(args, dev, stream, layers, ncopies, x_in, xs, ths, local, peers, tp, rank, world):
    """The step end to end through the C ABI (include/grinqh_b200.h) with host buffers:
    per step one pinned H2D of the step's activations (every linear's input, back to
    back), the four linears (grinqh_gemm_or_gemv; the row-parallel ones of a sharded
    layer through grinqh_gemv_allreduce for one row, grinqh_gemm_allreduce for 2..64
    rows, or followed by NCCL's all-reduce),
    all writing one output buffer, and one D2H of it. Returns (ms per step, max over
    ranks; H2D bytes; D2H bytes)."""
    from grinqh._ext import cabi, check, thresholds_arg, GRINQH_BF16, MODE_AUTO
    bits, M = args.bits, args.m
    lib = cabi()
    names = list(SHAPES)
    x_off, y_off, nx, ny = {}, {}, 0, 0
    for n in names:
        K, _ = local[n]
        x_off[n] = nx
        nx += M * K
    for n in names:
        y_off[n] = ny
        ny += M * local[n][1]
    host_x = torch.empty(nx, dtype=torch.bfloat16).pin_memory()
    for n in names:
        host_x[x_off[n]:x_off[n] + M * local[n][0]].copy_(x_in[n].reshape(-1).cpu())
    host_y = torch.empty(ny, dtype=torch.bfloat16).pin_memory()
    dev_x = torch.empty(nx, dtype=torch.bfloat16, device=dev)
    dev_y = torch.empty(ny, dtype=torch.bfloat16, device=dev)
    ws_bytes = max(max(lib.grinqh_workspace_size(M, K, N, bits, GROUP, MODE_AUTO),
                       lib.grinqh_allreduce_workspace_size(M, K, N, bits, GROUP, MODE_AUTO)) for K, N in local.values())
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev)  # tickets stay zero between calls
    th_args = {n: thresholds_arg(ths[n]) for n in names}
    workspace_zeroed = 0x100  # GRINQH_WORKSPACE_ZEROED
    h2d = host_x.numel() * host_x.element_size()
    d2h = host_y.numel() * host_y.element_size()
    if peers is not None:
        bufs = (ctypes.c_void_p * peers.world)(*peers.buffers)

    def e2e_step(c):
        dev_x.copy_(host_x, non_blocking=True)
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        for n in names:
            K, N = local[n]
            w, s = layers[c][n]
            xp, yp = dev_x.data_ptr() + 2 * x_off[n], dev_y.data_ptr() + 2 * y_off[n]
            if tp and n in ROW_PARALLEL and peers is not None and M == 1:
                check(lib.grinqh_gemv_allreduce(xp, GRINQH_BF16, K, w.data_ptr(), s.data_ptr(), None, bits, GROUP, N,
                                                th_args[n], yp, ws.data_ptr(), ws.numel(), peers.rank, peers.world,
                                                bufs, peers.n_cap, workspace_zeroed, st), f"e2e {n}")
                continue
            if tp and n in ROW_PARALLEL and peers is not None:
                check(lib.grinqh_gemm_allreduce(xp, GRINQH_BF16, M, K, w.data_ptr(), s.data_ptr(), None, bits, GROUP,
                                                N, th_args[n], MODE_AUTO | workspace_zeroed, yp, ws.data_ptr(),
                                                ws.numel(), peers.rank, peers.world, bufs, peers.n_cap, st),
                      f"e2e {n}")
                continue
            check(lib.grinqh_gemm_or_gemv(xp, GRINQH_BF16, M, K, w.data_ptr(), s.data_ptr(), None, bits, GROUP, N,
                                          th_args[n], MODE_AUTO | workspace_zeroed, yp, ws.data_ptr(), ws.numel(), st),
                  f"e2e {n}")
            if tp and n in ROW_PARALLEL:
                dist.all_reduce(dev_y[y_off[n]:y_off[n] + M * N])
        host_y.copy_(dev_y, non_blocking=True)

    with torch.cuda.stream(stream):
        e2e_step(0)
        torch.cuda.synchronize(dev)
        ge = []
        for c in range(ncopies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                e2e_step(c)
            ge.append(g)
        for i in range(3):
            ge[i % ncopies].replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        n_e2e = max(20, min(args.steps, 200))
        t_e = 0.0
        for i in range(n_e2e):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ge[i % ncopies].replay()
            b.record(stream)
            b.synchronize()  # the host reads the step's result
            t_e += a.elapsed_time(b)
    torch.cuda.synchronize(dev)
    del ge
    return max_over_ranks(t_e / n_e2e, dev, world), h2d, d2h


def grade_skew(bits, dev, stream, M=4096, K=4096, N=14336):
    """the opt-in per-token graded prefill (MODE_GRADED) at M = 4096, K = 4096,
    N = 14336 with unit-variance Student-t(3) activations, three threshold cases: every
    element in the lowest grade (zone 0 only), every element in the highest (all zones),
    and 70 / 20 / 10 % in grades 1 / 2 / 4. Per case: us per call, plane-MACs/s (2 N per
    active zone of every element) and the dense-equivalent 2 M N K TFLOP/s."""
    from grinqh.kernel import MODE_GRADED, grinqh_grade, grinqh_linear
    from grinqh.utils import pack_codes
    g = torch.Generator(device=dev).manual_seed(2)
    qmax = (1 << (bits - 1)) - 1
    w = torch.randn((K, N), generator=g, device=dev) * 0.02
    s = (w.view(K // GROUP, GROUP, N).abs().amax(1) / qmax).clamp_min(1e-8).to(torch.bfloat16)
    codes = torch.clamp(torch.round(w / s.float().repeat_interleave(GROUP, 0)), -qmax - 1, qmax).to(torch.int8)
    wp = pack_codes(codes, bits)
    del w, codes
    # Student-t(3) / sqrt(3): normal / sqrt(chi2_3 / 3), scaled to unit variance
    z = torch.randn((M, K), generator=g, device=dev)
    chi = torch.randn((M, K, 3), generator=g, device=dev).pow(2).sum(-1)
    x = (z / torch.sqrt(chi / 3) / math.sqrt(3.0)).to(torch.bfloat16)
    del z, chi
    a = x.abs().float().flatten()[:: 97].sort().values
    q70, q90 = float(a[int(0.7 * (a.numel() - 1))]), float(a[int(0.9 * (a.numel() - 1))])
    cases = {"lowest": [-1.0, float("inf"), float("inf"), float("inf")], "highest": [-1.0] * 4,
             "70_20_10": [-1.0, q70, q90, q90]}
    out = {}
    for name, th in cases.items():
        masks, _ = grinqh_grade(x, th, bits)
        mk = masks.to(torch.int32)
        zone_elems = int(sum(((mk >> zz) & 1).sum().item() for zz in range(bits // 2)))
        with torch.cuda.stream(stream):
            grinqh_linear(x, wp, s, None, bits, GROUP, N // 4, th, MODE_GRADED)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(3):
                grinqh_linear(x, wp, s, None, bits, GROUP, N // 4, th, MODE_GRADED)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / 3
        out[name] = {"us": round(us, 1), "plane_MAC_per_s": float("%.4g" % (N * zone_elems / (us * 1e-6))),
                     "dense_equiv_TFLOP/s": round(2 * M * N * K / us / 1e6, 1),
                     "zone_fill": round(zone_elems / (M * K * (bits // 2)), 4)}
    return out


def m_sweep(layers, bits, dev, stream, Ms=(16, 128, 1024, 8192)):
    """configs[1] sweep: each linear at M rows (dense path, as the reference runs rows
    > 1), two weight copies rotated; per (linear, M): us per call, weight-side bytes/s
    (packed planes + scales + x + y) and TFLOP/s (2 M N K)."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    g = torch.Generator(device=dev).manual_seed(11)
    out = {}
    for M in Ms:
        row = {}
        for name, (K, N) in SHAPES.items():
            x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
            R = 8 if M <= 1024 else 2
            with torch.cuda.stream(stream):
                for i in range(2):
                    w, s_ = layers[i % 2][name]
                    grinqh_gemm_or_gemv(x, w, s_, None, bits, GROUP, N // 4, [0.0] * 4)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for i in range(R):
                        w, s_ = layers[i % 2][name]
                        grinqh_gemm_or_gemv(x, w, s_, None, bits, GROUP, N // 4, [0.0] * 4)
                gr.replay()
                torch.cuda.synchronize(dev)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                gr.replay()
                gr.replay()
                b.record(stream)
            torch.cuda.synchronize(dev)
            us = a.elapsed_time(b) * 1e3 / (2 * R)
            nbytes = K * N * bits // 8 + (K // GROUP) * N * 2 + 2 * M * K + 2 * M * N
            row[name] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                         "TFLOP/s": round(2 * M * N * K / us / 1e6, 1)}
            del gr, x
        out[str(M)] = row
    return out


# ----------------------------------------------------------------------------- reference (CPU)
def _cpu_reference(args, steps_to_time, threads):
    """The reference's CPU path (restated with torch CPU ops in oracle/cpu_path.py) on
    the same workload: per step the four linears at M rows."""
    import oracle.cpu_path as CP
    from oracle import grinqh_oracle as O
    torch.set_num_threads(threads)
    bits, M = args.bits, args.m
    rng = np.random.default_rng(0)
    layer = {}
    for name, (K, N) in SHAPES.items():
        codes = rng.integers(-(1 << (bits - 1)), 1 << (bits - 1), size=(K, N)).astype(np.int8)
        packed = torch.from_numpy(O.pack_codes(codes, bits).view(np.int32))
        s = (torch.rand((K // GROUP, N)) * 1e-3).to(torch.bfloat16)
        x = torch.randn((M, K)).to(torch.bfloat16)
        th = torch.quantile(x.abs().float().flatten(), torch.tensor(QUANTILES)).tolist()
        layer[name] = (packed, s, x, th)
    total_bytes = 0
    for name, (K, N) in SHAPES.items():
        packed, s, x, th = layer[name]
        if M == 1:
            m = O.grade(x.float().numpy()[0], th, bits)
            planes = int(sum(((m >> z) & 1).sum() for z in range(bits // 2)))
            groups = int((m.reshape(K // GROUP, GROUP) != 0).any(1).sum())
        else:
            planes, groups = K * (bits // 2), K // GROUP
        total_bytes += planes * (N // 4) + groups * N * 2 + 2 * M * K + 2 * M * N

    def step():
        for name, (K, N) in SHAPES.items():
            packed, s, x, th = layer[name]
            CP.linear(x, packed, s, bits, GROUP, N // 4, th)

    step()  # warm-up
    t0 = time.perf_counter()
    for _ in range(steps_to_time):
        step()
    dt = (time.perf_counter() - t0) / steps_to_time
    return total_bytes / dt / 1e9, dt, total_bytes


def run_reference(args):
    threads = os.cpu_count() or 1
    steps = max(1, min(args.steps, 3))
    gbs, dt, nbytes = _cpu_reference(args, steps, threads)
    return {
        "impl": "reference",
        "metric": "quant-linear HBM GB/s, Llama-3-8B layer linears (qkv+o+gate_up+down), decode",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": 1, "steps": steps, "warmup": 1,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"configs[1] Llama-3-8B linear shapes, M={args.m}, b={args.bits}, group {GROUP}",
                   "algorithmic_bytes_per_step": nbytes,
                   "path": "reference CPU path restated in torch (oracle/cpu_path.py): M==1 masked-weight "
                           "oracle + fp32 matmul, M>1 eager dequant + matmul"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} full step(s) of the workload"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_only(args, dev):
    """One linear at --m rows (--graded: per-token graded, else the AUTO dispatch), called
    --warmup times and then --steps times eagerly on one GPU, two weight copies rotated
    (inputs larger than L2 between calls for the wide shapes). A short, fixed launch
    sequence for profiler captures (ncu -k ... -s <warmup> -c <n>); prints us per call."""
    from grinqh.kernel import grinqh_gemm_or_gemv
    from grinqh.utils import pack_codes
    name, bits, M = args.only, args.bits, args.m
    K, N = SHAPES[name]
    copies = []
    for seed in range(2):
        codes, s_ = make_codes(dev, bits, seed, name)
        copies.append((pack_codes(codes, bits), s_))
        del codes
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    th = torch.quantile(x.abs().float().flatten()[: 1 << 24], torch.tensor(QUANTILES, device=dev)).tolist()

    def call(i):
        w, s_ = copies[i % 2]
        if args.graded:
            return torch.ops.grinqh.linear(x, w, s_, None, bits, GROUP, N // 4, th, 2)
        return grinqh_gemm_or_gemv(x, w, s_, None, bits, GROUP, N // 4, th)

    for i in range(args.warmup):
        call(i)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.steps):
        call(i)
    b.record()
    torch.cuda.synchronize(dev)
    us = a.elapsed_time(b) * 1e3 / max(args.steps, 1)
    return {"only": name, "M": M, "bits": bits, "graded": bool(args.graded), "us_per_call": round(us, 2),
            "note": "eager calls for profiler captures; not a bench line"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", "--rows", dest="m", type=int, default=1,
                    help="decode batch rows per linear (--rows under torchrun, which claims --m)")
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the M = 16..8192 sweep of configs[1]")
    ap.add_argument("--replicas", action="store_true",
                    help="with several GPUs: independent replicas instead of the tensor-parallel layer")
    ap.add_argument("--only", choices=list(SHAPES), default=None,
                    help="profiling: call one linear at --m rows, --warmup then --steps times, and exit")
    ap.add_argument("--graded", action="store_true", help="with --only: per-token graded rows (mode 2)")
    args = ap.parse_args()
    if args.only:
        print(json.dumps(run_only(args, torch.device("cuda", 0))), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    if world > 1:
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    line = run_ours(args, rank, world, dev)
    if rank == 0:
        if not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            gbs, dt, _ = _cpu_reference(args, 1, threads)
            line["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                                    "sample": "1 full step of the workload (4 linears) on the host cores, "
                                              "reference CPU path restated in torch (oracle/cpu_path.py)"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
