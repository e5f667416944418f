"""Quantized-linear ops of the plugin, backed by the sm_100a CUDA library.

Mirrors the reference module ``grinqh/kernel.py``: importing it registers
``torch.ops.grinqh.gemm_or_gemv`` (same schema, kernel.py:646-657) and its fake
implementation for tracing (kernel.py:713-725), and exposes the same Python entry
points. There is no Triton, no Marlin and no CPU fallback: every function raises
on CPU tensors.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ._ext import MODE_AUTO, MODE_DENSE, MODE_GRADED, MODE_UNION, load_ops

load_ops()

__all__ = [
    "grinqh_gemm_or_gemv", "grinqh_linear", "grinqh_prefill_gemm_compiled", "grinqh_prefill_gemm",
    "grinqh_gemv_batch_union", "grinqh_prefill_marlin", "grinqh_grade", "grinqh_rmsnorm_grade",
    "grinqh_silu_mul_grade", "grinqh_gemv_batch_union_masked",
    "MODE_AUTO", "MODE_DENSE", "MODE_GRADED", "MODE_UNION",
]


def _out_shape(x: torch.Tensor, original_n: int):
    return x.shape[:-1] + (original_n * 4,)


@torch.library.register_fake("grinqh::gemm_or_gemv")
def _fake_gemm_or_gemv(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                       use_marlin=False):
    # kernel.py:713-725
    return torch.empty(_out_shape(x, original_n), device=x.device, dtype=x.dtype)


@torch.library.register_fake("grinqh::linear")
def _fake_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds, mode):
    return torch.empty(_out_shape(x, original_n), device=x.device, dtype=x.dtype)


@torch.library.register_fake("grinqh::pack")
def _fake_pack(words, max_bits):
    return words.new_empty((words.shape[0], (max_bits // 2) * (words.shape[1] // 4)))


@torch.library.register_fake("grinqh::pack_codes")
def _fake_pack_codes(codes, max_bits):
    return codes.new_empty((codes.shape[0], (max_bits // 2) * (codes.shape[1] // 16)), dtype=torch.uint32)


@torch.library.register_fake("grinqh::gemv_allreduce")
def _fake_gemv_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds, rank,
                         world, buffers, n_cap):
    return x.new_empty((*x.shape[:-1], 4 * original_n))


@torch.library.register_fake("grinqh::linear_allreduce")
def _fake_linear_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds, mode,
                           rank, world, buffers, cap):
    return x.new_empty((*x.shape[:-1], 4 * original_n))


@torch.library.register_fake("grinqh::unpack_checkpoint")
def _fake_unpack_checkpoint(src, max_bits, row0, rows, k0, dst, n_off):
    return None


@torch.library.register_fake("grinqh::unpack")
def _fake_unpack(packed, max_bits, original_n):
    return packed.new_empty((packed.shape[0], original_n * 4), dtype=torch.uint8)


@torch.library.register_fake("grinqh::grade")
def _fake_grade(x, thresholds, max_bits):
    return x.new_empty(x.shape, dtype=torch.uint8), x.new_empty((x.shape[-1],), dtype=torch.uint8)


@torch.library.register_fake("grinqh::rmsnorm_grade")
def _fake_rmsnorm_grade(x, residual, weight, eps, thresholds, max_bits):
    return (torch.empty_like(x), x.new_empty(x.shape, dtype=torch.uint8),
            x.new_empty((x.shape[-1],), dtype=torch.uint8))


@torch.library.register_fake("grinqh::silu_mul_grade")
def _fake_silu_mul_grade(x, thresholds, max_bits):
    shape = (*x.shape[:-1], x.shape[-1] // 2)
    return x.new_empty(shape), x.new_empty(shape, dtype=torch.uint8), x.new_empty((shape[-1],), dtype=torch.uint8)


@torch.library.register_fake("grinqh::union_linear_masked")
def _fake_union_linear_masked(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                              union_mask):
    return x.new_empty((*x.shape[:-1], 4 * original_n))


def grinqh_gemm_or_gemv(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                        bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                        thresholds: List[float], use_marlin: bool = False) -> torch.Tensor:
    """``y = x @ W (+ bias)`` with the reference dispatch (kernel.py:646-710): one row
    -> graded GEMV (thresholds apply), several rows -> dense ``x @ dtype(w * s)``.
    ``GRINQH_GRADED_PREFILL=1`` grades every row instead. ``use_marlin`` is ignored."""
    return torch.ops.grinqh.gemm_or_gemv(x, weight_packed, weight_scale, bias, max_bits, group_size,
                                         original_n, [float(t) for t in thresholds], use_marlin)


def grinqh_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                  mode: int = MODE_AUTO) -> torch.Tensor:
    """Explicit-mode entry: MODE_AUTO / MODE_DENSE / MODE_GRADED (every row graded by its
    own activations) / MODE_UNION (rows graded by max_m |x[m,k]|)."""
    return torch.ops.grinqh.linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                                   [float(t) for t in thresholds], int(mode))


def grinqh_prefill_gemm(x_flat, weight_packed, weight_scale, group_size, original_n, max_bits, bias=None):
    """Dense path ``x @ dtype(w * s)`` (kernel.py:561-587) for any number of rows."""
    return grinqh_linear(x_flat, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                         [0.0] * 4, MODE_DENSE)


def grinqh_prefill_gemm_compiled(x_flat, weight_packed, weight_scale, group_size, original_n, max_bits):
    """Same signature and numerics as the reference's torch.compile'd dense path
    (kernel.py:561-587); here a single CUDA kernel, nothing is compiled at run time."""
    return grinqh_prefill_gemm(x_flat, weight_packed, weight_scale, group_size, original_n, max_bits)


def grinqh_prefill_marlin(x_flat, weight_packed, weight_scale, group_size, original_n):
    """The reference's b=4 Marlin prefill (kernel.py:528-558) computes the dense W4A16
    product; this build has no Marlin and routes it to the dense kernel (max_bits=4)."""
    return grinqh_prefill_gemm(x_flat, weight_packed, weight_scale, group_size, original_n, 4)


def grinqh_gemv_batch_union(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                            bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                            thresholds: List[float]) -> torch.Tensor:
    """Small-batch GEMV graded by the row union max_m |x[m,k]| (kernel.py:607-643)."""
    return grinqh_linear(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds,
                         MODE_UNION)


def grinqh_grade(x: torch.Tensor, thresholds: List[float], max_bits: int):
    """Per-element zone masks (bit z: fp32|x| > t_z) and their union over rows."""
    return torch.ops.grinqh.grade(x, [float(t) for t in thresholds], max_bits)


def grinqh_rmsnorm_grade(x: torch.Tensor, residual: Optional[torch.Tensor], weight: Optional[torch.Tensor],
                         eps: float, thresholds: List[float], max_bits: int):
    """vLLM's RMSNorm (with the residual add when ``residual`` is given, updated in place)
    producing x for the next linear together with its grade masks and their union over
    rows: (out, masks, union)."""
    return torch.ops.grinqh.rmsnorm_grade(x, residual, weight, float(eps), [float(t) for t in thresholds], max_bits)


def grinqh_silu_mul_grade(x: torch.Tensor, thresholds: List[float], max_bits: int):
    """vLLM's SiluAndMul on x = [gate | up] with the grades of the product: (out, masks, union)."""
    return torch.ops.grinqh.silu_mul_grade(x, [float(t) for t in thresholds], max_bits)


def grinqh_gemv_batch_union_masked(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                                   bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                                   thresholds: List[float], union_mask: torch.Tensor) -> torch.Tensor:
    """grinqh_gemv_batch_union with the union of grades from the producer of x."""
    return torch.ops.grinqh.union_linear_masked(x, weight_packed, weight_scale, bias, max_bits, group_size,
                                                original_n, [float(t) for t in thresholds], union_mask)
