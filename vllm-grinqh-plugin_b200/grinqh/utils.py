"""Weight-layout helpers, mirroring the reference module ``grinqh/utils.py``.

``grinqh_input_preshuffle`` / ``grinqh_input_postshuffle`` are pure layout
permutations (torch views, any device). Packing and unpacking run on the GPU
through the sm_100a library and raise on CPU tensors.
"""
from __future__ import annotations

from enum import Enum
from typing import Union

import torch

from ._ext import load_ops

load_ops()


def grinqh_input_preshuffle(weight: torch.Tensor) -> torch.Tensor:
    """(K, 16, N/16) -> (K, N/16, 16) column permutation (utils.py:17-22)."""
    m, n = weight.shape
    assert n % 16 == 0, "N must be divisible by 16 for this layout."
    return weight.view(m, 16, n // 16).transpose(1, 2).contiguous().view(m, n)


def grinqh_input_postshuffle(weight: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`grinqh_input_preshuffle` (utils.py:25-30)."""
    m, n = weight.shape
    assert n % 16 == 0, "N must be divisible by 16 for this layout."
    return weight.view(m, n // 16, 16).transpose(1, 2).contiguous().view(m, n)


class BitLevel(Enum):
    """Number of 2-bit planes per weight (utils.py:33-37)."""
    TWO_BIT = 1
    FOUR_BIT = 2
    SIX_BIT = 3
    EIGHT_BIT = 4


def pack_cuda(A: torch.Tensor, max_bits: int = 8) -> torch.Tensor:
    """Bit-plane pack of preshuffled, shifted code words ``A`` (K, N/4) uint32
    -> (K, (b/2) * N/16) uint32, bit-exact with ``pack_triton`` (utils.py:125-146)."""
    if not A.is_cuda:
        raise AssertionError("GRINQH pack expects a CUDA tensor")
    if A.dtype not in (torch.uint32, torch.int32):
        raise AssertionError("GRINQH pack expects a uint32 tensor")
    return torch.ops.grinqh.pack(A.contiguous(), max_bits)


# the reference name (its tests and plugin call pack_triton)
pack_triton = pack_cuda


def pack_codes(codes: torch.Tensor, max_bits: int = 8) -> torch.Tensor:
    """Fused preshuffle + ``<< (8-b)`` + pack of int8 codes (K, N): the whole
    ``process_weights_after_loading`` transform (grinqh.py:202-211) in one kernel."""
    return torch.ops.grinqh.pack_codes(codes, max_bits)


def unpack_checkpoint(src: torch.Tensor, max_bits: int, row0: int, rows: int, k0: int, dst: torch.Tensor,
                      n_off: int) -> None:
    """One load-time kernel for a checkpoint shard (grinqh.py:154-168): unpack the
    compressed-tensors int32 weight ``src`` (rows = output features; int8 codes for
    b = 6), narrow it to rows ``[row0, row0 + rows)`` and columns
    ``[k0, k0 + dst.shape[0])``, and write the int8 codes transposed into
    ``dst[:, n_off:n_off + rows]``."""
    torch.ops.grinqh.unpack_checkpoint(src, max_bits, row0, rows, k0, dst, n_off)


def _bit_level(bit_level) -> int:
    return int(bit_level.value if isinstance(bit_level, BitLevel) else bit_level)


def unpack_pyt(B: torch.Tensor, row: Union[int, torch.Tensor], bit_level, original_n: int) -> torch.Tensor:
    """Rows of the packed tensor back to bytes ``shifted_code >> (8-b)`` (utils.py:149-177):
    returns (len(row), original_n) words of B's dtype, as the reference does."""
    b = 2 * _bit_level(bit_level)
    nz = b // 2
    n16 = original_n // 4
    if isinstance(row, int):
        row = torch.tensor([row], device=B.device)
    words = B.view(torch.int32) if B.dtype == torch.uint32 else B  # uint32 has no CUDA indexing kernel
    rows = words[row.to(B.device), : nz * n16].contiguous()
    out = torch.ops.grinqh.unpack(rows, b, original_n)
    return out.view(B.dtype if B.dtype in (torch.uint32, torch.int32) else torch.uint8).view(rows.shape[0], -1)


def unpack_triton(B: torch.Tensor, row: int, bit_level, original_n: int) -> torch.Tensor:
    """One row of :func:`unpack_pyt` as a flat tensor (utils.py:209-223)."""
    return unpack_pyt(B, int(row), bit_level, original_n).reshape(-1)
