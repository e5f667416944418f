"""The reference's CPU path, restated with torch CPU ops (test / baseline
infrastructure only: used by bench.py's ``cpu_baseline`` and ``--impl reference``
legs, never by the GPU path).

The reference itself cannot run on the GPU box's host (it is not shipped there),
and its GPU kernels are Triton. Its CPU-runnable path is plain torch:

* rows == 1: the test oracle ``get_masked_weight_ref`` + fp32 matmul
  (tests/test_grinqh_ops.py:28-55, 236-237), on weights unpacked from the planes
  by ``unpack_pyt`` + sign extension + ``grinqh_input_postshuffle``
  (grinqh/utils.py:149-177, 25-30);
* rows > 1: ``grinqh_prefill_gemm_compiled`` run eagerly (grinqh/kernel.py:561-587):
  unpack, sign-extend, postshuffle, ``w.to(dtype) * scale``, ``x @ w``.
"""
from __future__ import annotations

import torch

_SHIFTS = torch.tensor((6, 4, 2, 0), dtype=torch.int32)


def unpack_all(packed: torch.Tensor, max_bits: int, original_n: int) -> torch.Tensor:
    """unpack_pyt over every row (utils.py:149-177): (K, 4*original_n) uint8 bytes."""
    k = max_bits // 2
    n_zone = original_n // 4
    b = packed.view(torch.int32)
    planes = b[:, : n_zone * k].view(b.shape[0], k, n_zone)
    unpacked = (planes.unsqueeze(-1) >> _SHIFTS) & 0x03030303
    merge = (torch.arange(k, dtype=torch.int32) * 2).view(1, k, 1, 1).flip(1)
    res = (unpacked << merge).sum(dim=1, dtype=torch.int32)
    return res.view(b.shape[0], -1).view(torch.uint8)


def codes_from_packed(packed: torch.Tensor, max_bits: int, original_n: int) -> torch.Tensor:
    """kernel.py:571-576: sign-extended int8 codes in the original column order."""
    shift = 8 - max_bits
    u = unpack_all(packed, max_bits, original_n)
    w = (u.view(torch.int8) << shift) >> shift
    m, n = w.shape
    return w.view(m, n // 16, 16).transpose(1, 2).contiguous().view(m, n)


def masked_weight_ref(weight: torch.Tensor, x: torch.Tensor, thresholds, max_bits: int) -> torch.Tensor:
    """tests/test_grinqh_ops.py:28-55 (graded mask + mid-point bias, fp32 compare)."""
    shift_amt = 8 - max_bits
    x_abs = x.abs().float().flatten()
    w_u8 = (weight << shift_amt).view(torch.uint8)
    row_mask = torch.zeros_like(x_abs, dtype=torch.uint8)
    bias = torch.zeros_like(x_abs, dtype=torch.float32)
    bias_base = 1 << (max_bits - 1)
    prev = 0
    for zone in range(max_bits // 2):
        active = x_abs > thresholds[zone]
        row_mask |= active.to(torch.uint8) * (0xC0 >> 2 * zone)
        cur = bias_base >> (2 * zone + 2)
        bias += active * (cur - prev)
        prev = cur
    weight_masked = (w_u8 & row_mask[:, None]).view(torch.int8).float()
    return weight_masked / 2 ** shift_amt + bias[:, None]


def linear(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, max_bits: int, group_size: int,
           original_n: int, thresholds) -> torch.Tensor:
    """The reference's result for one linear, computed on the CPU."""
    w = codes_from_packed(packed, max_bits, original_n)
    if x.shape[0] == 1:
        wm = masked_weight_ref(w, x, thresholds, max_bits)
        y = x.float() @ (wm * scale.float().repeat_interleave(group_size, 0))
        return y.to(x.dtype)
    k, n = w.shape
    ws = (w.view(k // group_size, group_size, n).to(x.dtype) * scale.view(scale.shape[0], 1, n)).view(k, n)
    return x @ ws
