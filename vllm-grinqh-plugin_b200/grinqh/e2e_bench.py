"""End-to-end decode throughput of a GRINQH-quantized Llama in vLLM (random weights).

    python -m grinqh.e2e_bench [--tp N] [--batch 64] [--prompt 512] [--gen 256]
                               [--arch 8b|70b] [--max-bits 8] [--enforce-eager]
                               [--checkpoint DIR]

Builds a local model directory with the Llama-3 architecture's config.json (8B:
hidden 4096, FFN 14336, 32 layers, 32 / 8 heads; 70B: 8192, 28672, 80, 64 / 8;
vocab 128256) whose ``quantization_config`` names ``grinqh``, and a
``GRINQH_JSON_PATH`` threshold file for every quantized linear. vLLM loads it with
``load_format="dummy"`` (random weights: the staged int32 codes keep whatever bits
the allocation holds, the bf16 scales are uniform in [-1e-3, 1e-3]); every
``LinearBase`` of the model goes through this plugin (process_weights_after_loading
packs the planes on the GPU; apply calls torch.ops.grinqh.gemm_or_gemv). Prompts are
uniform random token ids, generation is greedy with ``ignore_eos`` so every sequence
produces exactly ``--gen`` tokens.

With ``--checkpoint DIR`` it runs a checkpoint written by ``python -m grinqh.quantize``
(real codes, scales and calibrated thresholds from its config) instead of the random
model.

Reported (one JSON line): output tokens / second over the whole generate call, the
decode-only rate (generate time minus a prefill-only call with one output token),
and the times. The plugin reaches vLLM's worker processes through an entry-point
file (``vllm.general_plugins: grinqh = grinqh:register``) written next to the model
directory and put on ``PYTHONPATH``, so nothing is installed.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

ARCH = {
    "8b": dict(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
               num_key_value_heads=8),
    "70b": dict(hidden_size=8192, intermediate_size=28672, num_hidden_layers=80, num_attention_heads=64,
                num_key_value_heads=8),
}


def write_model(root: str, arch: str, max_bits: int, layers: int | None) -> str:
    cfg = dict(ARCH[arch])
    if layers:
        cfg["num_hidden_layers"] = layers
    cfg.update({
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": 128256,
        "max_position_embeddings": 8192, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
        "torch_dtype": "bfloat16", "bos_token_id": 128000, "eos_token_id": 128001,
        "tie_word_embeddings": False, "hidden_act": "silu",
        "quantization_config": {
            "quant_method": "grinqh",
            "grinqh": {"max_bits": max_bits},
            "config_groups": {"group_0": {"weights": {"num_bits": max_bits, "group_size": 128}}},
        },
    })
    model_dir = os.path.join(root, f"llama3-{arch}-grinqh")
    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    # one threshold set per quantized linear, keyed by vLLM module name
    th = {}
    for i in range(cfg["num_hidden_layers"]):
        for name in ("self_attn.qkv_proj", "self_attn.o_proj", "mlp.gate_up_proj", "mlp.down_proj"):
            th[f"model.layers.{i}.{name}"] = [0.02, 0.05, 0.1, 0.2]
    th_path = os.path.join(root, "thresholds.json")
    with open(th_path, "w") as f:
        json.dump({"thresholds": th}, f)
    os.environ["GRINQH_JSON_PATH"] = th_path
    return model_dir


def expose_plugin(root: str) -> None:
    """An entry-point file that vLLM's plugin loader finds through importlib.metadata
    in this process and in the worker processes it starts."""
    site = os.path.join(root, "site")
    info = os.path.join(site, "grinqh_b200-0.1.dist-info")
    os.makedirs(info, exist_ok=True)
    with open(os.path.join(info, "METADATA"), "w") as f:
        f.write("Metadata-Version: 2.1\nName: grinqh-b200\nVersion: 0.1\n")
    with open(os.path.join(info, "entry_points.txt"), "w") as f:
        f.write("[vllm.general_plugins]\ngrinqh = grinqh:register\n")
    paths = [site, PKG_DIR] + [p for p in os.environ.get("PYTHONPATH", "").split(os.pathsep) if p]
    os.environ["PYTHONPATH"] = os.pathsep.join(paths)
    sys.path[:0] = [site, PKG_DIR]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--arch", choices=sorted(ARCH), default="8b")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (0: the architecture's)")
    ap.add_argument("--max-bits", type=int, default=8)
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.6)
    ap.add_argument("--enforce-eager", action="store_true")
    ap.add_argument("--checkpoint", default=None, help="a GRINQH checkpoint directory (grinqh.quantize)")
    args = ap.parse_args()

    root = tempfile.mkdtemp(prefix="grinqh_e2e_")
    if args.checkpoint:
        model_dir, load_format = args.checkpoint, "auto"
        with open(os.path.join(model_dir, "config.json")) as f:
            vocab = json.load(f)["vocab_size"]
    else:
        model_dir, load_format, vocab = write_model(root, args.arch, args.max_bits, args.layers), "dummy", 128256
    expose_plugin(root)

    import numpy as np
    from vllm import LLM, SamplingParams

    llm = LLM(model=model_dir, quantization="grinqh", load_format=load_format, tensor_parallel_size=args.tp,
              skip_tokenizer_init=True, dtype="bfloat16", max_model_len=args.prompt + args.gen + 16,
              gpu_memory_utilization=args.gpu_memory_utilization, enforce_eager=args.enforce_eager, seed=0)
    rng = np.random.default_rng(0)
    prompts = [{"prompt_token_ids": rng.integers(0, vocab, args.prompt).tolist()} for _ in range(args.batch)]
    gen = SamplingParams(max_tokens=args.gen, min_tokens=args.gen, ignore_eos=True, temperature=0.0,
                         detokenize=False)
    one = SamplingParams(max_tokens=1, ignore_eos=True, temperature=0.0, detokenize=False)
    llm.generate(prompts[:2], SamplingParams(max_tokens=8, ignore_eos=True, temperature=0.0, detokenize=False),
                 use_tqdm=False)  # warm-up
    t0 = time.perf_counter()
    llm.generate(prompts, one, use_tqdm=False)
    t_prefill = time.perf_counter() - t0
    t0 = time.perf_counter()
    outs = llm.generate(prompts, gen, use_tqdm=False)
    t_all = time.perf_counter() - t0
    n_out = sum(len(o.outputs[0].token_ids) for o in outs)
    decode_tokens = n_out - args.batch
    line = {
        "metric": "decode tok/s, Llama GRINQH in vLLM (" + ("checkpoint" if args.checkpoint else "random weights") + ")",
        "arch": args.checkpoint or args.arch, "layers": args.layers or ARCH[args.arch]["num_hidden_layers"],
        "tp": args.tp,
        "batch": args.batch, "prompt": args.prompt, "gen": args.gen, "max_bits": args.max_bits,
        "output_tokens": n_out, "generate_s": round(t_all, 3), "prefill_s": round(t_prefill, 3),
        "output_tok_per_s": round(n_out / t_all, 1),
        "decode_tok_per_s": round(decode_tokens / max(t_all - t_prefill, 1e-9), 1),
        "enforce_eager": args.enforce_eager,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
