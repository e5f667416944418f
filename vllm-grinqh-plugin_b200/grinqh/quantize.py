"""Offline quantizer and threshold calibrator: a Hugging Face Llama-family checkpoint ->
a GRINQH checkpoint that the plugin loads (the reference ships neither; its README
expects a compressed-tensors pack-quantized model plus a GRINQH_JSON_PATH file).

    python -m grinqh.quantize --model DIR --out DIR [--bits 8] [--group 128]
                              [--calib-tokens 2048] [--calib-seq 512]
                              [--quantiles 0.2,0.4,0.6,0.8] [--device cuda] [--seed 0]

Weights: every ``{q,k,v,o,gate,up,down}_proj`` of the decoder layers is quantized by
symmetric round-to-nearest per (output row, group of ``group`` input columns):
``s = absmax / (2^(b-1) - 1)`` rounded to the checkpoint dtype (never below 1e-8),
``code = clamp(rint(w / s), -2^(b-1), 2^(b-1) - 1)``. They are stored in the
compressed-tensors pack-quantized layout the plugin's loader reads
(grinqh/grinqh.py:154-168): ``weight_packed`` int32 (N, K*b/32) written by
compressed-tensors' own ``pack_to_int32``, ``weight_scale`` (N, K/group) and
``weight_shape``; for b = 6, ``weight`` int8 (N, K) as the reference expects
(grinqh/grinqh.py:131-132). Every other tensor is copied unchanged.

Thresholds: the model runs on ``calib_tokens`` uniformly random token ids (or ids from
``--calib-file``, one integer per whitespace-separated token); forward hooks record
|x| entering q_proj, o_proj, gate_proj and down_proj of every layer, which are the
inputs of vLLM's qkv_proj, o_proj, gate_up_proj and down_proj. The thresholds of a
module are the given quantiles of those values (at most ``max_samples`` of them,
drawn uniformly), keyed by vLLM module name. They go into the config
(``quantization_config.grinqh.thresholds``) and into ``grinqh_thresholds.json`` for
``GRINQH_JSON_PATH``.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
from typing import Dict, Iterable, List, Optional

import numpy as np
import torch

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
# HF module whose input is the input of a vLLM module (merged q/k/v and gate/up share it)
CALIB_SOURCES = {"self_attn.q_proj": "self_attn.qkv_proj", "self_attn.o_proj": "self_attn.o_proj",
                 "mlp.gate_proj": "mlp.gate_up_proj", "mlp.down_proj": "mlp.down_proj"}


def rtn_quantize(w: torch.Tensor, bits: int, group: int, dtype: torch.dtype = torch.bfloat16):
    """(N, K) weight -> int8 codes (N, K) and scales (N, K/group) in ``dtype``."""
    n, k = w.shape
    if k % group:
        raise ValueError(f"input features {k} are not a multiple of the group size {group}")
    qmax = (1 << (bits - 1)) - 1
    wf = w.float().reshape(n, k // group, group)
    s = (wf.abs().amax(dim=2) / qmax).clamp_min(1e-8).to(dtype)
    q = torch.round(wf / s.float().unsqueeze(2)).clamp(-(1 << (bits - 1)), qmax)
    return q.reshape(n, k).to(torch.int8), s


def pack_checkpoint_weight(codes: torch.Tensor, bits: int) -> Dict[str, torch.Tensor]:
    """The tensors of one quantized linear, by suffix, in the layout the loader reads."""
    if bits == 6:
        return {"weight": codes.cpu()}
    from compressed_tensors.compressors.pack_quantized.helpers import pack_to_int32
    return {"weight_packed": pack_to_int32(codes.cpu(), bits)}


class _Recorder:
    """|x| samples entering a module, at most ``max_samples`` kept, uniformly drawn."""

    def __init__(self, max_samples: int, gen: torch.Generator):
        self.max_samples = max_samples
        self.gen = gen
        self.chunks: List[torch.Tensor] = []
        self.seen = 0

    def add(self, x: torch.Tensor) -> None:
        a = x.detach().abs().float().reshape(-1)
        self.seen += a.numel()
        per_call = max(1, self.max_samples // 16)
        if a.numel() > per_call:
            idx = torch.randint(0, a.numel(), (per_call,), generator=self.gen, device="cpu").to(a.device)
            a = a[idx]
        self.chunks.append(a.cpu())

    def quantiles(self, qs: Iterable[float]) -> List[float]:
        v = torch.cat(self.chunks).numpy()
        if v.size > self.max_samples:
            v = np.random.default_rng(0).choice(v, self.max_samples, replace=False)
        return [float(t) for t in np.quantile(v.astype(np.float64), list(qs))]


def calibrate(model: torch.nn.Module, input_ids: torch.Tensor, quantiles: Iterable[float],
              max_samples: int = 1 << 22, batch_rows: int = 4) -> Dict[str, List[float]]:
    """Thresholds keyed by vLLM module name (``model.layers.{i}.self_attn.qkv_proj`` ...)."""
    gen = torch.Generator().manual_seed(0)
    recorders: Dict[str, _Recorder] = {}
    hooks = []
    for name, mod in model.named_modules():
        for src, dst in CALIB_SOURCES.items():
            if name.endswith("." + src) and ".layers." in name:
                vname = name[: -len(src)] + dst
                rec = recorders.setdefault(vname, _Recorder(max_samples, gen))
                hooks.append(mod.register_forward_pre_hook(lambda m, args, rec=rec: rec.add(args[0])))
    try:
        with torch.no_grad():
            for i in range(0, input_ids.shape[0], batch_rows):
                model(input_ids=input_ids[i:i + batch_rows])
    finally:
        for h in hooks:
            h.remove()
    qs = list(quantiles)
    return {name: rec.quantiles(qs) for name, rec in sorted(recorders.items())}


def _is_target(name: str) -> bool:
    parts = name.split(".")
    return len(parts) >= 3 and parts[-1] == "weight" and parts[-2] in PROJ and ".layers." in name


def quantize_model(model_dir: str, out_dir: str, bits: int = 8, group: int = 128, calib_tokens: int = 2048,
                   calib_seq: int = 512, quantiles: Iterable[float] = (0.2, 0.4, 0.6, 0.8),
                   device: Optional[str] = None, seed: int = 0, calib_ids: Optional[torch.Tensor] = None,
                   max_shard_bytes: int = 4 << 30) -> Dict[str, List[float]]:
    from safetensors.torch import save_file
    from transformers import AutoConfig, AutoModelForCausalLM

    if bits not in (2, 4, 6, 8):
        raise ValueError(f"bits must be 2, 4, 6 or 8 (got {bits})")
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    cfg = AutoConfig.from_pretrained(model_dir)
    td = str(getattr(cfg, "torch_dtype", None) or getattr(cfg, "dtype", None) or "bfloat16")
    dtype = torch.float16 if td.replace("torch.", "") == "float16" else torch.bfloat16  # scales and activations
    model = AutoModelForCausalLM.from_pretrained(model_dir, torch_dtype=dtype).to(device).eval()

    # ---- thresholds
    if calib_ids is None:
        g = torch.Generator().manual_seed(seed)
        rows = max(1, calib_tokens // calib_seq)
        calib_ids = torch.randint(0, cfg.vocab_size, (rows, min(calib_seq, calib_tokens)), generator=g)
    thresholds = calibrate(model, calib_ids.to(device), quantiles)

    # ---- weights
    os.makedirs(out_dir, exist_ok=True)
    state = model.state_dict()
    shards: List[Dict[str, torch.Tensor]] = [{}]
    size = 0
    for name, t in state.items():
        if _is_target(name):
            codes, s = rtn_quantize(t, bits, group, dtype)
            base = name[: -len(".weight")]
            out = {f"{base}.{k}": v for k, v in pack_checkpoint_weight(codes, bits).items()}
            out[f"{base}.weight_scale"] = s.cpu()
            out[f"{base}.weight_shape"] = torch.tensor(list(t.shape), dtype=torch.int64)
        else:
            out = {name: t.detach().cpu().contiguous()}
        for k, v in out.items():
            nbytes = v.numel() * v.element_size()
            if size + nbytes > max_shard_bytes and shards[-1]:
                shards.append({})
                size = 0
            shards[-1][k] = v.contiguous()
            size += nbytes
    weight_map = {}
    for i, sh in enumerate(shards):
        fname = "model.safetensors" if len(shards) == 1 else f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(out_dir, fname), metadata={"format": "pt"})
        weight_map.update({k: fname for k in sh})
    if len(shards) > 1:
        with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": weight_map}, f, indent=1)

    # ---- config and thresholds
    conf = cfg.to_dict()
    conf["quantization_config"] = {
        "quant_method": "grinqh",
        "format": "pack-quantized",
        "grinqh": {"max_bits": bits, "thresholds": thresholds},
        "config_groups": {"group_0": {"targets": ["Linear"], "weights": {
            "num_bits": bits, "group_size": group, "type": "int", "symmetric": True, "strategy": "group"}}},
        "ignore": ["lm_head"],
    }
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(conf, f, indent=1)
    with open(os.path.join(out_dir, "grinqh_thresholds.json"), "w") as f:
        json.dump({"thresholds": thresholds}, f, indent=1)
    for extra in ("generation_config.json", "tokenizer.json", "tokenizer_config.json", "special_tokens_map.json",
                  "tokenizer.model"):
        p = os.path.join(model_dir, extra)
        if os.path.exists(p):
            shutil.copy(p, os.path.join(out_dir, extra))
    return thresholds


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--bits", type=int, default=8)
    ap.add_argument("--group", type=int, default=128)
    ap.add_argument("--calib-tokens", type=int, default=2048)
    ap.add_argument("--calib-seq", type=int, default=512)
    ap.add_argument("--calib-file", default=None, help="whitespace-separated token ids")
    ap.add_argument("--quantiles", default="0.2,0.4,0.6,0.8")
    ap.add_argument("--device", default=None)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    ids = None
    if args.calib_file:
        with open(args.calib_file) as f:
            flat = torch.tensor([int(t) for t in f.read().split()], dtype=torch.long)
        n = flat.numel() // args.calib_seq * args.calib_seq
        ids = flat[:n].reshape(-1, args.calib_seq) if n else flat[None]
    th = quantize_model(args.model, args.out, args.bits, args.group, args.calib_tokens, args.calib_seq,
                        [float(q) for q in args.quantiles.split(",")], args.device, args.seed, ids)
    print(json.dumps({"out": args.out, "bits": args.bits, "group": args.group, "modules": len(th)}))


if __name__ == "__main__":
    main()
