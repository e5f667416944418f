"""Peer buffers for the fused row-parallel linear (torch.ops.grinqh.gemv_allreduce).

Every tensor-parallel rank allocates one device buffer with the library
(``grinqh_allreduce_buffer_alloc``, zeroed), the ranks exchange its CUDA IPC handle
over a process group, and each rank opens the others' buffers, so that the kernel can
store its partial sums straight into every rank's buffer over NVLink. One
:class:`PeerBuffers` serves every row-parallel layer of a model (the calls on a stream
are ordered, and every rank makes the same calls in the same order).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from ._ext import cabi


def _check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"GRINQH {what}: {cabi().grinqh_last_error().decode()}")


class PeerBuffers:
    """This rank's buffer and the mapped buffers of the other ranks of ``group``.

    ``n_cap``: the widest output (N) the buffers serve. Collective: every rank of the
    group must construct it together (it exchanges handles and ends with a barrier),
    on the device that will run the kernel."""

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
