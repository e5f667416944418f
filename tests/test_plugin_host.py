"""Host logic of the vLLM plugin surface, on CPU: config parsing, threshold lookup,
shard ids, and the tensor-parallel weight loader (fake layers carrying tp_rank)."""
import json

import numpy as np
import pytest
import torch

import oracle as O


@pytest.fixture()
def plugin(monkeypatch):
    import vllm.model_executor.parameter as P
    from grinqh import grinqh as G
    state = {"rank": 0, "size": 1}
    monkeypatch.setattr(P, "get_tensor_model_parallel_rank", lambda: state["rank"])
    monkeypatch.setattr(P, "get_tensor_model_parallel_world_size", lambda: state["size"])
    G._tp_state = state
    return G


def _cfg(**grinqh_extra):
    return {"config_groups": {"group_0": {"weights": {"num_bits": 4, "group_size": 128}}},
            "grinqh": {"thresholds": {"model.layers.0.mlp.down_proj": [0.1, 0.2]}, **grinqh_extra}}


def test_register_is_idempotent():
    import grinqh
    grinqh.register()
    grinqh.register()
    from vllm.model_executor.layers.quantization import get_quantization_config
    from grinqh.grinqh import GRINQHConfig
    assert get_quantization_config("grinqh") is GRINQHConfig


def test_from_config_reads_checkpoint(plugin, monkeypatch):
    monkeypatch.delenv("GRINQH_JSON_PATH", raising=False)
    c = plugin.GRINQHConfig.from_config(_cfg())
    assert c.num_bits == 4 and c.group_size == 128
    assert c.get_name() == "GRINQH"
    assert c.get_min_capability() == 100
    assert c.get_config_filenames() == []
    assert torch.bfloat16 in c.get_supported_act_dtypes()
    c2 = plugin.GRINQHConfig.from_config(_cfg(max_bits=8))  # grinqh.max_bits wins (grinqh.py:82)
    assert c2.num_bits == 8
    assert plugin.GRINQHConfig.override_quantization_method({}, "grinqh") == "grinqh"
    assert plugin.GRINQHConfig.override_quantization_method({}, "awq") is None


def test_json_path_overrides(plugin, monkeypatch, tmp_path):
    p = tmp_path / "th.json"
    p.write_text(json.dumps({"thresholds": {"a.qkv_proj": [1, 2, 3, 4]}}))
    monkeypatch.setenv("GRINQH_JSON_PATH", str(p))
    c = plugin.GRINQHConfig.from_config(_cfg())
    assert c.thresholds == {"a.qkv_proj": [1, 2, 3, 4]}


def test_missing_thresholds_raise(plugin, monkeypatch):
    monkeypatch.delenv("GRINQH_JSON_PATH", raising=False)
    with pytest.raises(ValueError, match="no 'grinqh.thresholds'"):
        plugin.GRINQHConfig.from_config({"grinqh": {}})
    with pytest.raises(ValueError, match="max_bits"):
        plugin.GRINQHConfig(thresholds={}, max_bits=3)


def test_get_quant_method_pads_and_raises(plugin):
    from vllm.model_executor.layers.linear import LinearBase
    c = plugin.GRINQHConfig(thresholds={"l.down_proj": [0.5, 0.25]}, max_bits=4)
    layer = LinearBase.__new__(LinearBase)
    m = c.get_quant_method(layer, "l.down_proj")
    assert isinstance(m, plugin.GRINQHLinearMethod)
    assert m.layer_thresholds == [0.5, 0.25, 0.0, 0.0]
    with pytest.raises(ValueError, match="no thresholds for layer"):
        c.get_quant_method(layer, "l.up_proj")
    assert c.get_quant_method(torch.nn.Linear(2, 2), "x") is None


def test_shard_ids(plugin):
    assert plugin._resolve_shard_id(None) == 0
    assert plugin._resolve_shard_id(2) == 2
    assert [plugin._resolve_shard_id(s) for s in ("q", "k", "v", "gate", "up")] == [0, 1, 2, 0, 1]
    with pytest.raises(ValueError, match="unsupported shard_id"):
        plugin._resolve_shard_id("o")


def _make_layer(plugin, bits, k_local, parts, k_full, rank, size, kv_replicas=1):
    plugin._tp_state.update(rank=rank, size=size)
    layer = torch.nn.Module()
    layer.tp_rank, layer.tp_size = rank, size
    layer.num_kv_head_replicas = kv_replicas
    cfg = plugin.GRINQHConfig(thresholds={}, max_bits=bits)
    m = plugin.GRINQHLinearMethod(cfg, [0.0] * 4)
    m.create_weights(layer, k_local, parts, k_full, sum(parts) * size, torch.bfloat16)
    return layer, m


def _ckpt(codes_nk, bits):
    """checkpoint tensors for one shard, (N, K) orientation (compressed-tensors)."""
    if bits == 6:
        return torch.from_numpy(codes_nk.copy())
    return torch.from_numpy(O.ct_pack_to_int32(codes_nk, bits))


@pytest.mark.parametrize("bits", [4, 6, 8])
@pytest.mark.parametrize("rank,size", [(0, 1), (1, 2), (3, 4)])
def test_loader_column_parallel_merged(plugin, bits, rank, size):
    """gate/up (MergedColumnParallelLinear): each rank keeps its N slice of each shard."""
    rng = np.random.default_rng(bits * 10 + rank)
    K, n_gate, G = 256, 128, 128
    lim = 1 << (bits - 1)
    full = {s: rng.integers(-lim, lim, size=(n_gate, K)).astype(np.int8) for s in ("gate", "up")}
    scl = {s: rng.standard_normal((n_gate, K // G)).astype(np.float32) for s in ("gate", "up")}
    nl = n_gate // size
    layer, _ = _make_layer(plugin, bits, K, [nl, nl], K, rank, size)
    wp = getattr(layer, layer.grinqh_weight_param_name)
    for s in ("gate", "up"):
        wp.weight_loader(wp, _ckpt(full[s], bits), s)
        layer.weight_scale.weight_loader(layer.weight_scale, torch.from_numpy(scl[s]).to(torch.bfloat16), s)
    got = wp.data.view(torch.int8).numpy()
    exp = np.concatenate([full[s][rank * nl:(rank + 1) * nl].T for s in ("gate", "up")], axis=1)
    np.testing.assert_array_equal(got, exp)
    exp_s = np.concatenate([scl[s][rank * nl:(rank + 1) * nl].T for s in ("gate", "up")], axis=1)
    np.testing.assert_array_equal(layer.weight_scale.data.float().numpy(),
                                  torch.from_numpy(exp_s).to(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("rank,size", [(0, 2), (1, 2), (2, 4)])
def test_loader_row_parallel(plugin, rank, size):
    """o/down (RowParallelLinear): each rank keeps its K slice (codes and scale groups)."""
    rng = np.random.default_rng(7 + rank)
    N, K, G, bits = 64, 512, 128, 8
    codes = rng.integers(-128, 128, size=(N, K)).astype(np.int8)
    scl = rng.standard_normal((N, K // G)).astype(np.float32)
    kl = K // size
    layer, _ = _make_layer(plugin, bits, kl, [N], K, rank, size)
    wp = layer.weight_packed
    wp.weight_loader(wp, _ckpt(codes, bits))
    layer.weight_scale.weight_loader(layer.weight_scale, torch.from_numpy(scl).to(torch.bfloat16))
    np.testing.assert_array_equal(wp.data.view(torch.int8).numpy(), codes[:, rank * kl:(rank + 1) * kl].T)
    gl = kl // G
    np.testing.assert_array_equal(layer.weight_scale.data.float().numpy(),
                                  torch.from_numpy(scl[:, rank * gl:(rank + 1) * gl].T.copy()).to(torch.bfloat16).float().numpy())


def test_loader_qkv_replicated_kv_heads(plugin):
    """QKV at tp 4 with 2 KV heads: k/v slices repeat every 2 ranks."""
    rng = np.random.default_rng(3)
    K, hd = 128, 16
    q_full = rng.integers(-128, 128, size=(8 * hd, K)).astype(np.int8)
    k_full = rng.integers(-128, 128, size=(2 * hd, K)).astype(np.int8)
    rank, size = 3, 4
    layer, _ = _make_layer(plugin, 8, K, [2 * hd, hd, hd], K, rank, size, kv_replicas=2)
    wp = layer.weight_packed
    wp.weight_loader(wp, _ckpt(q_full, 8), "q")
    wp.weight_loader(wp, _ckpt(k_full, 8), "k")
    wp.weight_loader(wp, _ckpt(k_full, 8), "v")
    got = wp.data.view(torch.int8).numpy()
    np.testing.assert_array_equal(got[:, :2 * hd], q_full[rank * 2 * hd:(rank + 1) * 2 * hd].T)
    kv_rank = rank // 2
    np.testing.assert_array_equal(got[:, 2 * hd:3 * hd], k_full[kv_rank * hd:(kv_rank + 1) * hd].T)


def test_loader_rejects_bad_shapes(plugin):
    with pytest.raises(ValueError, match="divisible by 16"):
        _make_layer(plugin, 8, 128, [40], 128, 0, 1)
    with pytest.raises(ValueError, match="multiple of group_size"):
        _make_layer(plugin, 8, 100, [64], 100, 0, 1)
    layer, _ = _make_layer(plugin, 8, 128, [32], 256, 1, 2)
    with pytest.raises(ValueError, match="does not fit"):
        layer.weight_packed.weight_loader(layer.weight_packed, _ckpt(np.zeros((32, 192), np.int8), 8))
