"""The offline quantizer / calibrator (grinqh.quantize) on a tiny random Llama, on
CPU: the written checkpoint is in the compressed-tensors layout the plugin loads, its
codes and scales are this build's RTN of the original weights (checked with the CPU
oracle's codec and quantizer), and the thresholds are the requested quantiles of the
activations entering each vLLM module."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as O

transformers = pytest.importorskip("transformers")


def tiny_llama(tmp_path, dtype=torch.bfloat16):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=512, max_position_embeddings=256, tie_word_embeddings=False)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(dtype)
    d = os.path.join(tmp_path, "src")
    model.save_pretrained(d)
    return d, model


@pytest.mark.parametrize("bits", [4, 8, 6])
def test_quantized_checkpoint_layout_codes_and_thresholds(tmp_path, bits):
    from safetensors.torch import load_file
    from grinqh.quantize import quantize_model, rtn_quantize
    src, model = tiny_llama(str(tmp_path))
    out = os.path.join(str(tmp_path), "out")
    ids = torch.randint(0, 512, (2, 64), generator=torch.Generator().manual_seed(1))
    th = quantize_model(src, out, bits=bits, group=128, device="cpu", calib_ids=ids)
    tensors = load_file(os.path.join(out, "model.safetensors"))
    sd = model.state_dict()
    for i in range(2):
        for proj in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                     "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            base = f"model.layers.{i}.{proj}"
            w = sd[base + ".weight"]
            assert base + ".weight_packed" in tensors or bits == 6
            assert tuple(tensors[base + ".weight_shape"].tolist()) == tuple(w.shape)
            if bits == 6:
                codes = tensors[base + ".weight"].numpy()
            else:
                packed = tensors[base + ".weight_packed"]
                assert packed.dtype == torch.int32 and packed.shape == (w.shape[0], w.shape[1] * bits // 32)
                codes = O.ct_unpack_from_int32(packed.numpy(), bits, w.shape)
            # the oracle's RTN on the (K, N) orientation gives the same codes and scales
            want_codes, want_s = O.rtn_quantize(w.float().numpy().T, bits, 128, "bf16")
            np.testing.assert_array_equal(codes, want_codes.T)
            s = tensors[base + ".weight_scale"]
            assert s.dtype == torch.bfloat16 and s.shape == (w.shape[0], w.shape[1] // 128)
            np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), want_s.T)
            c2, s2 = rtn_quantize(w, bits, 128)
            np.testing.assert_array_equal(c2.numpy(), codes)
    # every other tensor is copied unchanged
    for name in ("model.embed_tokens.weight", "lm_head.weight", "model.norm.weight"):
        assert torch.equal(tensors[name], sd[name])
    # thresholds: four vLLM modules per layer, increasing, the quantiles of the inputs
    assert sorted(th) == sorted(f"model.layers.{i}.{m}" for i in range(2)
                                for m in ("self_attn.qkv_proj", "self_attn.o_proj", "mlp.gate_up_proj",
                                          "mlp.down_proj"))
    for v in th.values():
        assert len(v) == 4 and all(a <= b for a, b in zip(v, v[1:])) and v[0] > 0
    seen = {}
    hook = model.model.layers[0].mlp.down_proj.register_forward_pre_hook(
        lambda m, a: seen.setdefault("x", []).append(a[0].detach().abs().float().reshape(-1)))
    with torch.no_grad():
        for r in range(ids.shape[0]):
            model(input_ids=ids[r:r + 1])
    hook.remove()
    allx = torch.cat(seen["x"]).numpy().astype(np.float64)
    np.testing.assert_allclose(th["model.layers.0.mlp.down_proj"], np.quantile(allx, [0.2, 0.4, 0.6, 0.8]),
                               rtol=0.05)
    # the config and the JSON are what the plugin reads
    with open(os.path.join(out, "config.json")) as f:
        qc = json.load(f)["quantization_config"]
    assert qc["quant_method"] == "grinqh" and qc["grinqh"]["max_bits"] == bits
    from grinqh.grinqh import GRINQHConfig
    os.environ.pop("GRINQH_JSON_PATH", None)
    c = GRINQHConfig.from_config(qc)
    assert c.num_bits == bits and c.group_size == 128 and c.thresholds == th
    with open(os.path.join(out, "grinqh_thresholds.json")) as f:
        assert json.load(f)["thresholds"] == th
