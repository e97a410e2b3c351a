"""Tensor-parallel row sums over NVLink peer memory.

The decoder's row-parallel projections (o_proj and the FFN down projection)
end in a sum over the tensor-parallel ranks, and in the decode step that sum
is followed by the residual add and the next RMSNorm.  ``PeerSumNorm`` does
all three in one kernel (``cq_peer_sum_norm``, csrc/cq_peer.cu): every rank
owns a region of device memory that every other rank maps through CUDA IPC,
a projection GEMM writes its part straight into the region, and the kernel
reads the parts of all ranks over NVLink (peer loads, no copy engine, no
NCCL) after a flag handshake in the same regions.  The reference has no
multi-device path; this is the build's own.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._tensors import cq_dtype, stream_ptr

FLAG_BYTES = 256  # the region's flag words; part buffers follow


class PeerSumNorm:
    """Peer-memory regions for ``rows`` x ``dim`` parts of ``dtype`` on every
    rank of ``group`` (at most 8 ranks), mapped by every rank.  Collective:
    every rank of the group constructs it at the same point."""

    def __init__(self, group, rows: int, dim: int, dtype=torch.bfloat16, device=None):
        import torch.distributed as dist
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 1 <= self.world <= 8:
            raise ValueError("PeerSumNorm: 1 to 8 ranks")
        if dim % 8:
            raise ValueError("PeerSumNorm: dim must be a multiple of 8")
        self.rows, self.dim, self.dtype = rows, dim, dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib()
        self.part_bytes = (rows * dim * torch.finfo(dtype).bits // 8 + 15) // 16 * 16
        nbytes = int(lib.cq_peer_region_bytes(self.part_bytes))
        self.region = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)  # zeroed before any peer maps it
        handles = [None] * self.world
        dist.all_gather_object(handles, self.region.untyped_storage()._share_cuda_(), group=group)
        self._mapped = []  # peer storages, kept open while this object lives
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.region.data_ptr())
            else:
                st = torch.UntypedStorage._new_shared_cuda(*h)
                self._mapped.append(st)
                ptrs.append(st.data_ptr())
        self.ptrs = (ctypes.c_uint64 * self.world)(*ptrs)
        self.counter = torch.zeros(2, dtype=torch.int64, device=self.device)
        dist.barrier(group=group)  # every rank has mapped every region before the first call

    def part(self, parity: int, rows: int | None = None) -> torch.Tensor:
        """This rank's part buffer ``parity`` as a [rows, dim] tensor (a view
        of the region: write the projection's output here, e.g. with
        ``torch.matmul(..., out=part)``)."""
        rows = self.rows if rows is None else rows
        off = FLAG_BYTES + parity * self.part_bytes
        n = rows * self.dim * torch.finfo(self.dtype).bits // 8
        return self.region[off:off + n].view(self.dtype).view(rows, self.dim)

    def __call__(self, x: torch.Tensor, w: torch.Tensor, eps: float, y: torch.Tensor, parity: int) -> None:
        """x <- x + (sum over ranks of part ``parity``), y <- RMSNorm(x) * w,
        for the rows of x ([rows, dim], contiguous, this rank's copy)."""
        rows = x.shape[0]
        _lib.check(_lib.lib().cq_peer_sum_norm(self.ptrs, self.world, self.rank, parity, self.part_bytes, rows,
                                               self.dim, x.data_ptr(), w.data_ptr(), float(eps), y.data_ptr(),
                                               self.counter.data_ptr(), cq_dtype(x), stream_ptr(x.device)),
                   "peer_sum_norm")
