"""vLLM quantization plugin surface of GRINQH (mirrors the reference ``grinqh/grinqh.py``).

``@register_quantization_config("grinqh")`` registers :class:`GRINQHConfig`;
every ``LinearBase`` gets a :class:`GRINQHLinearMethod` whose ``apply`` calls
``torch.ops.grinqh.gemm_or_gemv`` (the sm_100a kernels). Differences from the
reference, all on purpose:

* tensor parallelism: the weight loader narrows checkpoint tensors to this rank
  (output rows for column-parallel layers, input columns for row-parallel ones),
  where the reference refuses ``tp_size > 1`` (grinqh.py:128-129);
* load-time packing is one fused CUDA kernel (preshuffle + shift + pack);
* there is no Marlin: ``layer.grinqh_use_marlin`` is always False;
* minimum capability is 100 (sm_100a only).
"""
from __future__ import annotations

import json
import os
from typing import List, Optional

import torch
from compressed_tensors import unpack_from_int32
from torch.nn.parameter import Parameter
from vllm.logger import init_logger
from vllm.model_executor import PackedvLLMParameter
from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig, QuantizeMethodBase
from vllm.model_executor.layers.quantization.utils.layer_utils import replace_parameter
from vllm.model_executor.utils import set_weight_attrs

from . import allreduce as _allreduce  # noqa: F401  (registers torch.ops.grinqh.row_parallel_linear)
from .kernel import grinqh_gemm_or_gemv  # noqa: F401  (registers torch.ops.grinqh)
from .utils import pack_codes, unpack_checkpoint

logger = init_logger("vllm.grinqh")

# merged-layer shard ids (grinqh.py:31)
_SHARD_IDS = {"q": 0, "k": 1, "v": 2, "gate": 0, "up": 1}


def _resolve_shard_id(shard_id) -> int:
    """grinqh.py:34-42: None for non-merged layers, ints pass through, names map."""
    if shard_id is None:
        return 0
    if isinstance(shard_id, int):
        return shard_id
    if shard_id in _SHARD_IDS:
        return _SHARD_IDS[shard_id]
    raise ValueError(f"GRINQH: unsupported shard_id {shard_id!r}")


def shard_rank_for(layer, shard_id, tp_rank: int) -> int:
    """Rank index of this rank's slice of a checkpoint shard. k/v of a QKV layer
    with replicated KV heads (tp_size > num_kv_heads) repeat every
    ``num_kv_head_replicas`` ranks."""
    if shard_id in ("k", "v"):
        return tp_rank // int(getattr(layer, "num_kv_head_replicas", 1) or 1)
    return tp_rank


def checkpoint_row0(rows_total: int, out_rows: int, out_rank: int) -> int:
    """First checkpoint row of this rank's slice (the row narrowing of
    :func:`narrow_checkpoint`)."""
    if rows_total == out_rows:
        return 0
    if rows_total < (out_rank + 1) * out_rows:
        raise ValueError(f"GRINQH: checkpoint shard has {rows_total} rows, rank slice {out_rank} of "
                         f"{out_rows} does not fit")
    return out_rank * out_rows


def narrow_checkpoint(t: torch.Tensor, out_rows: int, out_rank: int, in_cols: Optional[int], in_rank: int):
    """Narrow a checkpoint tensor in (N, K) orientation to this rank: rows
    ``[out_rank*out_rows, +out_rows)`` when the tensor holds more rows than the
    rank owns (column parallel), columns ``[in_rank*in_cols, +in_cols)`` when it
    holds more columns (row parallel)."""
    if t.shape[0] != out_rows:
        if t.shape[0] < (out_rank + 1) * out_rows:
            raise ValueError(f"GRINQH: checkpoint shard has {t.shape[0]} rows, rank slice {out_rank} of "
                             f"{out_rows} does not fit")
        t = t.narrow(0, out_rank * out_rows, out_rows)
    if in_cols is not None and t.shape[1] != in_cols:
        if t.shape[1] < (in_rank + 1) * in_cols:
            raise ValueError(f"GRINQH: checkpoint has {t.shape[1]} input columns, rank slice {in_rank} of "
                             f"{in_cols} does not fit")
        t = t.narrow(1, in_rank * in_cols, in_cols)
    return t


@register_quantization_config("grinqh")
class GRINQHConfig(QuantizationConfig):
    """GRINQH quantization config (grinqh.py:45-115)."""

    def __init__(self, thresholds: dict[str, list[float]], max_bits: int = 8, group_size: int = 128):
        super().__init__()
        if max_bits not in (2, 4, 6, 8):
            raise ValueError(f"GRINQH: max_bits must be 2, 4, 6 or 8, got {max_bits}")
        self.thresholds = thresholds
        self.num_bits = max_bits
        self.group_size = group_size

    def get_name(self) -> str:
        return "GRINQH"

    def get_supported_act_dtypes(self) -> list:
        return [torch.float16, torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def override_quantization_method(cls, hf_quant_cfg, user_quant, hf_config=None):
        if user_quant == "grinqh":
            return "grinqh"
        return None

    @classmethod
    def from_config(cls, config: dict) -> "GRINQHConfig":
        """grinqh.py:78-101: bits from ``grinqh.max_bits`` or compressed-tensors'
        ``config_groups.group_0.weights.num_bits``; thresholds from the file named by
        ``GRINQH_JSON_PATH`` (key ``thresholds``) or ``grinqh.thresholds``."""
        group_0_weights = config.get("config_groups", {}).get("group_0", {}).get("weights", {})
        grinqh_cfg = config.get("grinqh", {})
        num_bits = grinqh_cfg.get("max_bits", group_0_weights.get("num_bits", 8))
        group_size = group_0_weights.get("group_size", 128)
        json_path = os.environ.get("GRINQH_JSON_PATH")
        if json_path is not None:
            logger.warning("GRINQH: GRINQH_JSON_PATH is set, overriding checkpoint thresholds with %s", json_path)
            with open(json_path) as f:
                thresholds = json.load(f)["thresholds"]
        elif "thresholds" in grinqh_cfg:
            thresholds = grinqh_cfg["thresholds"]
        else:
            raise ValueError("GRINQH: checkpoint quantization_config has no 'grinqh.thresholds'. Calibrate the "
                             "model first or set GRINQH_JSON_PATH.")
        return cls(thresholds=thresholds, max_bits=num_bits, group_size=group_size)

    def get_quant_method(self, layer: torch.nn.Module, prefix: str) -> QuantizeMethodBase | None:
        if isinstance(layer, LinearBase):
            t_vals = self.thresholds.get(prefix)
            if t_vals is None:
                raise ValueError(f"GRINQH: no thresholds for layer '{prefix}'. Thresholds must be keyed by vLLM "
                                 "module names (e.g. qkv_proj).")
            t_vals = (list(t_vals) + [0.0] * 4)[:4]  # pad to 4 in lower <8 bit settings
            return GRINQHLinearMethod(self, t_vals, layer_name=prefix)
        return None


class GRINQHLinearMethod(LinearMethodBase):
    """create_weights / process_weights_after_loading / apply (grinqh.py:118-249)."""

    PACK_FACTOR = 4  # int8 codes per int32 of the staging parameter

    def __init__(self, quant_config: GRINQHConfig, layer_thresholds: List[float] = None,
                 layer_name: str = "unknown"):
        super().__init__()
        self.quant_config = quant_config
        self.layer_thresholds = layer_thresholds
        self.layer_name = layer_name

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size,
                       output_size, params_dtype, **extra_weight_attrs):
        num_bits = self.quant_config.num_bits
        group = self.quant_config.group_size
        n_local = sum(output_partition_sizes)
        k_local = input_size_per_partition
        if n_local % 16:
            raise ValueError(f"GRINQH: output features per rank ({n_local}) must be divisible by 16")
        if k_local % group:
            raise ValueError(f"GRINQH: input features per rank ({k_local}) must be a multiple of group_size {group}")
        tp_rank = int(getattr(layer, "tp_rank", 0) or 0)
        row_parallel = k_local != input_size
        in_rank = tp_rank if row_parallel else 0
        param_name = "weight" if num_bits == 6 else "weight_packed"
        parts = list(output_partition_sizes)

        def grinqh_weight_loader(param, loaded_weight, shard_id=None):
            shard = _resolve_shard_id(shard_id)
            merged = len(parts) > 1
            out_rows = parts[shard] if merged else n_local
            n_off = sum(parts[:shard]) if merged else 0
            out_rank = shard_rank_for(layer, shard_id, tp_rank)
            if param is scales:
                # (N, K/g) in the checkpoint -> this rank's (K_local/g, N slice)
                s = narrow_checkpoint(loaded_weight, out_rows, out_rank, k_local // group, in_rank)
                param.data[:, n_off:n_off + out_rows].copy_(s.to(param.device).T)
                return
            if param.data.is_cuda:
                # one kernel: unpack + rank narrowing + transposed copy into the staging codes
                src = loaded_weight.to(param.device)
                row0 = checkpoint_row0(src.shape[0], out_rows, out_rank)
                k0 = 0 if input_size == k_local else in_rank * k_local
                if k0 + k_local > input_size:
                    raise ValueError(f"GRINQH: checkpoint has {input_size} input columns, rank slice {in_rank} of "
                                     f"{k_local} does not fit")
                unpack_checkpoint(src, num_bits, row0, out_rows, k0, param.data.view(torch.int8), n_off)
                return
            w = loaded_weight.to(param.device)
            if num_bits != 6:  # b=6 checkpoints store int8 codes (grinqh.py:151-153)
                w = unpack_from_int32(w, num_bits, torch.Size((w.shape[0], input_size)))
            w = narrow_checkpoint(w, out_rows, out_rank, k_local, in_rank)
            param.data.view(torch.int8)[:, n_off:n_off + out_rows].copy_(w.T.to(torch.int8))

        weight = PackedvLLMParameter(
            data=torch.empty(k_local, n_local // self.PACK_FACTOR, dtype=torch.int32),
            input_dim=0, output_dim=1, packed_dim=1, packed_factor=self.PACK_FACTOR,
            weight_loader=grinqh_weight_loader,
        )
        layer.register_parameter(param_name, weight)
        layer.grinqh_weight_param_name = param_name

        scales = Parameter(torch.empty(k_local // group, n_local, dtype=params_dtype), requires_grad=False)
        layer.register_parameter("weight_scale", scales)
        set_weight_attrs(scales, {"weight_loader": grinqh_weight_loader})

        weight_shape = Parameter(torch.empty(2, dtype=torch.int64), requires_grad=False)
        set_weight_attrs(weight_shape, {"weight_loader": lambda p, w, shard_id=None: None})
        layer.register_parameter("weight_shape", weight_shape)

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        """Codes (K, N) int8 -> bit planes (K, (b/2)*N/16) uint32 in one CUDA kernel
        (grinqh.py:202-212: preshuffle, << (8-b), pack_triton)."""
        param = getattr(layer, layer.grinqh_weight_param_name)
        codes = param.data.view(torch.int8)
        layer.original_n = codes.shape[1] // self.PACK_FACTOR
        packed = pack_codes(codes, max_bits=self.quant_config.num_bits)
        replace_parameter(layer, layer.grinqh_weight_param_name, packed)
        layer.grinqh_use_marlin = False
        # GRINQH_FUSED_ALLREDUCE=1: a row-parallel layer whose output vLLM would
        # all-reduce does the reduction itself (grinqh.allreduce.row_parallel_linear:
        # one row in one GEMV + NVLink-sum kernel, 2..64 rows in one skinny GEMM +
        # NVLink-sum kernel). Layers built with
        # reduce_results=False (the model reduces elsewhere) are left alone.
        layer.grinqh_fused_allreduce = False
        if (os.environ.get("GRINQH_FUSED_ALLREDUCE") == "1" and hasattr(layer, "input_is_parallel")
                and getattr(layer, "reduce_results", False) and int(getattr(layer, "tp_size", 1) or 1) > 1):
            layer.reduce_results = False
            layer.grinqh_fused_allreduce = True
            # the peer buffers are set up here, at load time (collective over the TP
            # group, same layer order on every rank), never inside graph capture
            from .allreduce import FUSED_MAX_ROWS, tp_peers
            tp_peers(packed.device, FUSED_MAX_ROWS * 4 * layer.original_n)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        if getattr(layer, "grinqh_fused_allreduce", False):
            # vLLM passes the bias on rank 0 only; the fused op adds the full bias once
            full_bias = None if getattr(layer, "skip_bias_add", False) else getattr(layer, "bias", None)
            return torch.ops.grinqh.row_parallel_linear(
                x, getattr(layer, layer.grinqh_weight_param_name), layer.weight_scale, full_bias,
                self.quant_config.num_bits, self.quant_config.group_size, layer.original_n,
                list(self.layer_thresholds))
        return torch.ops.grinqh.gemm_or_gemv(
            x,
            getattr(layer, layer.grinqh_weight_param_name),
            layer.weight_scale,
            bias,
            self.quant_config.num_bits,
            self.quant_config.group_size,
            layer.original_n,
            self.layer_thresholds,
            layer.grinqh_use_marlin,
        )
