"""Tensor-parallel row sums over NVLink peer memory.

The decoder's row-parallel projections (o_proj and the FFN down projection)
end in a sum over the tensor-parallel ranks, and in the decode step that sum
is followed by the residual add and the next RMSNorm.  ``PeerSumNorm`` does
all three in one kernel (``cq_peer_sum_norm``, csrc/cq_peer.cu): every rank
allocates a region of device memory, maps every other rank's region through
CUDA IPC in its own device context, and the kernel pushes this rank's part
into every region over NVLink, waits on flags in its own region and sums the
parts there (no copy engine, no NCCL).  The reference has no multi-device
path; this is the build's own.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._tensors import cq_dtype, stream_ptr

MAX_ROWS = 64


class PeerSumNorm:
    """Peer-memory regions for parts of up to ``rows`` x ``dim`` values on
    every rank of ``group`` (at most 8 ranks, rows at most 64).  Collective:
    every rank of the group constructs it, and calls it and ``close`` in the
    same order."""

    def __init__(self, group, rows: int, dim: int, device=None):
        import torch.distributed as dist
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 1 <= self.world <= 8 or not 1 <= rows <= MAX_ROWS or dim % 8:
            raise ValueError("PeerSumNorm: 1-8 ranks, 1-64 rows and dim a multiple of 8")
        self.rows, self.dim = rows, dim
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib()
        nbytes = int(lib.cq_peer_region_bytes(rows, dim, self.world))
        self._own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.cq_peer_region_alloc(nbytes, ctypes.byref(self._own), handle), "PeerSumNorm")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        with torch.cuda.device(self.device):  # peer regions mapped into this rank's device context
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own.value)
                    continue
                p = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(h, 64)
                _lib.check(lib.cq_peer_region_open(buf, ctypes.byref(p)), "PeerSumNorm")
                self._opened.append(p)
                ptrs.append(p.value)
        self.ptrs = (ctypes.c_uint64 * self.world)(*ptrs)
        self.counter = torch.zeros(2, dtype=torch.int64, device=self.device)
        dist.barrier(group=group)  # every rank has mapped every region before the first call

    def __call__(self, part: torch.Tensor, x: torch.Tensor, w: torch.Tensor, eps: float, y: torch.Tensor,
                 parity: int) -> None:
        """x <- x + (sum over the ranks of their ``part``), y <- RMSNorm(x) *
        w, for the rows of x ([rows, dim] contiguous, this rank's copy;
        ``part`` this rank's [rows, dim]).  ``parity`` alternates between
        consecutive calls."""
        if self.ptrs is None:
            raise RuntimeError("PeerSumNorm: closed")
        rows = x.shape[0]
        if (x.dim() != 2 or tuple(part.shape) != tuple(x.shape) or tuple(y.shape) != tuple(x.shape)
                or x.shape[1] != self.dim or not 1 <= rows <= self.rows or w.numel() != self.dim):
            raise ValueError(f"PeerSumNorm: part, x, y must be [rows <= {self.rows}, {self.dim}] and w [{self.dim}]")
        if len({part.dtype, x.dtype, y.dtype, w.dtype}) != 1 or not x.is_contiguous() or not y.is_contiguous():
            raise ValueError("PeerSumNorm: part, x, y, w of one dtype; x and y contiguous")
        part = part if part.is_contiguous() else part.contiguous()
        _lib.check(_lib.lib().cq_peer_sum_norm(self.ptrs, self.world, self.rank, parity, self.rows, rows, self.dim,
                                               part.data_ptr(), x.data_ptr(), w.data_ptr(), float(eps), y.data_ptr(),
                                               self.counter.data_ptr(), cq_dtype(x), stream_ptr(x.device)),
                   "peer_sum_norm")

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (collective: no rank
        frees its region while another may still write into it)."""
        import torch.distributed as dist
        if self.ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.cq_peer_region_close(p)
            dist.barrier(group=self.group)
            lib.cq_peer_region_free(self._own)
        self._opened, self.ptrs = [], None
