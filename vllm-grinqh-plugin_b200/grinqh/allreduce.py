"""Peer buffers for the fused row-parallel linear (torch.ops.grinqh.gemv_allreduce for
one row, torch.ops.grinqh.linear_allreduce for one graded row or 2..64 dense rows).

Every tensor-parallel rank allocates one device buffer with the library
(``grinqh_allreduce_buffer_alloc``, zeroed), the ranks exchange its CUDA IPC handle
over a process group, and each rank opens the others' buffers, so that the kernel can
store its partial sums straight into every rank's buffer over NVLink. One
:class:`PeerBuffers` serves every row-parallel layer of a model (the calls on a stream
are ordered, and every rank makes the same calls in the same order).
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ._ext import cabi


def _check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"GRINQH {what}: {cabi().grinqh_last_error().decode()}")


class PeerBuffers:
    """This rank's buffer and the mapped buffers of the other ranks of ``group``.

    ``n_cap``: the largest output (rows x columns, M * N) one call writes. Collective:
    every rank of the group must construct it together (it exchanges handles and ends
    with a barrier), on the device that will run the kernel."""

    def __init__(self, group: Optional[dist.ProcessGroup], n_cap: int, device: Optional[torch.device] = None):
        lib = cabi()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("GRINQH fused all-reduce supports at most 8 ranks")
        self.n_cap = int(n_cap)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            nbytes = lib.grinqh_allreduce_buffer_bytes(self.world, self.n_cap)
            if nbytes == 0:
                raise ValueError("GRINQH fused all-reduce: invalid world size or n_cap")
            own = ctypes.c_void_p()
            _check(lib.grinqh_allreduce_buffer_alloc(nbytes, ctypes.byref(own)), "peer buffer allocation")
            self._own = own.value
            handle = (ctypes.c_ubyte * 64)()
            _check(lib.grinqh_ipc_get_handle(ctypes.c_void_p(self._own), handle), "IPC handle")
            handles: List[bytes] = [b""] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.buffers: List[int] = []
            self._opened: List[int] = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.buffers.append(self._own)
                    continue
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                p = ctypes.c_void_p()
                _check(lib.grinqh_ipc_open_handle(hb, ctypes.byref(p)), f"opening rank {r}'s buffer")
                self.buffers.append(p.value)
                self._opened.append(p.value)
        dist.barrier(group=group)

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's (after a barrier,
        so that no rank still writes into it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = cabi()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.grinqh_ipc_close_handle(ctypes.c_void_p(p))
            lib.grinqh_allreduce_buffer_free(ctypes.c_void_p(self._own))
        self._own = None
        self._opened = []


def gemv_allreduce(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                   bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                   thresholds, peers: PeerBuffers) -> torch.Tensor:
    """y = sum over the ranks of (this rank's K slice of x) @ W_rank, for one row,
    identical on every rank; ``bias`` (the full bias, on every rank) is added once."""
    return torch.ops.grinqh.gemv_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                                           list(thresholds), peers.rank, peers.world, peers.buffers, peers.n_cap)


def linear_allreduce(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                     bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                     thresholds, peers: PeerBuffers, mode: int = 0) -> torch.Tensor:
    """As :func:`gemv_allreduce` for x of shape [..., K]: one graded row or 2..64 dense
    rows (mode as torch.ops.grinqh.linear; 0 = AUTO). Other shapes raise a
    RuntimeError containing "fused all-reduce not supported" before any launch."""
    return torch.ops.grinqh.linear_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                                             list(thresholds), mode, peers.rank, peers.world, peers.buffers,
                                             peers.n_cap)


# ----------------------------------------------------------------------------- vLLM
# One set of peer buffers per device, over vLLM's tensor-parallel group, created by
# the first fused call (vLLM's profiling forward, before any CUDA-graph capture; every
# rank runs that forward, so the collective setup lines up).
_TP_PEERS: Dict[int, PeerBuffers] = {}
# Rows the fused kernels take (one graded row; up to this many dense rows).
FUSED_MAX_ROWS = 64


def tp_peers(device: torch.device, n_cap: int) -> PeerBuffers:
    """The device's peer buffers, grown (collectively: every rank makes the same calls)
    when a call writes more values (M * N) than they hold. The replaced buffers are
    closed, so growth must not happen while a captured CUDA graph still uses them: it
    is refused during capture (the first forward, before any capture, sizes them for
    FUSED_MAX_ROWS rows of the layer's width)."""
    from vllm.distributed import get_tp_group
    key = torch.device(device).index or 0
    p = _TP_PEERS.get(key)
    if p is None or p.n_cap < n_cap:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GRINQH fused all-reduce: peer buffers must be sized before CUDA-graph capture "
                               f"(need {n_cap} values)")
        if p is not None:
            p.close()
        p = PeerBuffers(get_tp_group().cpu_group, max(int(n_cap), 8192), device)
        _TP_PEERS[key] = p
    return p


def fused_row_supported(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                        original_n: int, group_size: int) -> bool:
    """The fused kernel takes one row of x, the single-row GEMV's shapes, 8-byte aligned
    packed weights and 4-byte aligned scales (grinqh_gemv_allreduce refuses the rest;
    a shape whose launch plan does not fit is refused by the call itself)."""
    n = 4 * original_n
    return (x.numel() == weight_packed.shape[0] and n % 32 == 0 and group_size % 4 == 0
            and weight_packed.shape[0] % group_size == 0 and weight_packed.data_ptr() % 8 == 0
            and weight_scale.data_ptr() % 4 == 0)


def fused_rows_supported(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                         original_n: int, group_size: int) -> bool:
    """2..FUSED_MAX_ROWS dense rows: the skinny GEMM's shapes (N % 64, K and group_size
    multiples of 32) and alignments (x and the packed weights 16-byte, scales 4-byte)."""
    k = weight_packed.shape[0]
    m = x.numel() // max(k, 1)
    return (2 <= m <= FUSED_MAX_ROWS and x.shape[-1] == k and (4 * original_n) % 64 == 0 and k % 32 == 0
            and group_size % 32 == 0 and k % group_size == 0 and x.data_ptr() % 16 == 0
            and weight_packed.data_ptr() % 16 == 0 and weight_scale.data_ptr() % 4 == 0)


@torch.library.custom_op("grinqh::row_parallel_linear", mutates_args=())
def row_parallel_linear(x: torch.Tensor, weight_packed: torch.Tensor, weight_scale: torch.Tensor,
                        bias: Optional[torch.Tensor], max_bits: int, group_size: int, original_n: int,
                        thresholds: List[float]) -> torch.Tensor:
    """A row-parallel linear with its tensor-parallel sum: ``bias`` is the full bias
    (added once). One row: the fused graded GEMV + NVLink sum; 2..64 rows: the fused
    dense skinny GEMM + NVLink sum; more rows: the GEMM followed by vLLM's all-reduce
    (RowParallelLinear.forward), bias on rank 0 only. Opaque to the compiler, so the
    branch on the row count is taken at run time (the same on every rank)."""
    from vllm.distributed import get_tensor_model_parallel_rank, tensor_model_parallel_all_reduce
    one = fused_row_supported(x, weight_packed, weight_scale, original_n, group_size)
    if one or fused_rows_supported(x, weight_packed, weight_scale, original_n, group_size):
        peers = tp_peers(x.device, FUSED_MAX_ROWS * 4 * original_n)
        try:
            if one:
                return gemv_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                                      thresholds, peers)
            return linear_allreduce(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n,
                                    thresholds, peers)
        except RuntimeError as e:  # refused before launch (every rank refuses alike): unfused path
            if "fused all-reduce not supported" not in str(e):
                raise
    rank_bias = bias if get_tensor_model_parallel_rank() == 0 else None
    y = torch.ops.grinqh.gemm_or_gemv(x, weight_packed, weight_scale, rank_bias, max_bits, group_size, original_n,
                                      thresholds, False)
    return tensor_model_parallel_all_reduce(y)


@row_parallel_linear.register_fake
def _(x, weight_packed, weight_scale, bias, max_bits, group_size, original_n, thresholds):
    return x.new_empty((*x.shape[:-1], 4 * original_n))
