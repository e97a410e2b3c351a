"""One long sequence over several GPUs: sequence-split attention.

The reference runs on one device and has no multi-device path; this module
is the build's own (no reference counterpart).  A sequence whose compressed
cache does not fit, or whose decode should be spread, is cut into contiguous
token ranges, one per rank.  Every range starts at a multiple of
lcm(stride_k, stride_v), so it starts on an I-frame of both components: each
rank's compressed shard is exactly the matching slice of the unsplit cache
(anchors never cross a boundary, cache.py:99-116), and the last rank -- the
tail owner -- is the one that appends new tokens.

Each rank attends the queries over its own shard (``local_partials``) and
gets fp32 partial outputs with their natural-log log-sum-exp.  One
all-gather over the process group (NCCL over NVLink on GPUs, gloo on CPU for
the protocol tests) brings every rank's partials to every rank
(``exchange_partials``), and ``cq_lse_merge`` combines them on the device
(``merge_partials``):

    out = sum_i exp(lse_i - M) o_i / sum_i exp(lse_i - M),   M = max_i lse_i

For a query chunk (q_len > 1) the chunk's own tokens must sit in the tail
shard: the causal mask (anchored at the end of the keys, attention.py:8-20)
applies there, and every other shard's keys precede all queries and are
attended without a mask.  ``sequence_parallel_attention`` checks this on
every rank (one tiny all-reduce of the tail shard's length) and raises on all
of them when the tail shard holds fewer than q_len tokens (short sequences,
where ``shard_bounds`` can leave the tail short or empty).  The messages are
small (B*Hq*q_len*(D+1) floats per rank), so the exchange is latency-bound
rather than bandwidth-bound.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .trace import traced
from ._tensors import cq_dtype, require_cuda, stream_ptr


def shard_bounds(T: int, world: int, stride_k: int, stride_v: int) -> list[tuple[int, int]]:
    """Token range [start, end) of each of ``world`` ranks for a sequence of
    ``T`` tokens: contiguous, in rank order, every start a multiple of
    lcm(stride_k, stride_v), the last range ending at T (the tail owner).
    Ranges may be empty when T is short."""
    if world < 1 or T < 0 or stride_k < 1 or stride_v < 1:
        raise ValueError("shard_bounds: need world >= 1, T >= 0 and positive strides")
    align = stride_k * stride_v // math.gcd(stride_k, stride_v)
    units = -(-T // align)
    per = -(-units // world) if units else 0
    out = []
    for r in range(world):
        lo = min(r * per * align, T)
        hi = T if r == world - 1 else min((r + 1) * per * align, T)
        out.append((lo, hi))
    return out


def local_partials(queries: torch.Tensor, cache, scale: float, tail: bool):
    """This rank's partial attention over its shard: (o fp32 [B, Hq, Tq, D],
    lse fp32 [B, Hq, Tq]).  ``tail``: this rank owns the newest tokens (the
    causal mask applies when q_len > 1).  An empty shard contributes nothing
    (lse = -inf)."""
    from .attention import chronoquant_sdpa_with_lse
    B, Hq, Tq, D = queries.shape
    if cache.offset == 0:
        return (torch.zeros((B, Hq, Tq, D), dtype=torch.float32, device=queries.device),
                torch.full((B, Hq, Tq), -math.inf, dtype=torch.float32, device=queries.device))
    return chronoquant_sdpa_with_lse(queries, cache, scale, causal=tail or Tq == 1)


@traced("cq.seq_exchange")
def exchange_partials(o: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather every rank's partials: (o [world, ...], lse [world, ...]),
    rank-major.  Every rank calls it with the same shapes, in the same order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    os_ = [torch.empty_like(o) for _ in range(world)]
    ls_ = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(os_, o.contiguous(), group=group)
    dist.all_gather(ls_, lse.contiguous(), group=group)
    return torch.stack(os_), torch.stack(ls_)


@traced("cq.seq_merge")
def merge_partials(o_all: torch.Tensor, lse_all: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
    """Combine gathered partials on the device with cq_lse_merge (CUDA only:
    there is no host fallback).  o_all: [parts, ..., D] fp32, lse_all:
    [parts, ...] fp32."""
    require_cuda(o_all, lse_all)
    if o_all.dtype != torch.float32 or lse_all.dtype != torch.float32:
        raise ValueError("merge_partials: partials must be fp32")
    parts, D = o_all.shape[0], o_all.shape[-1]
    if tuple(lse_all.shape) != tuple(o_all.shape[:-1]):
        raise ValueError("merge_partials: lse shape must be o shape without the head dim")
    o_all, lse_all = o_all.contiguous(), lse_all.contiguous()
    out = torch.empty(o_all.shape[1:], dtype=out_dtype, device=o_all.device)
    rows = out.numel() // D
    _lib.check(_lib.lib().cq_lse_merge(lse_all.data_ptr(), o_all.data_ptr(), parts, rows, D, out.data_ptr(),
                                       cq_dtype(out), stream_ptr(o_all.device)), "merge_partials")
    return out


def sequence_parallel_attention(queries: torch.Tensor, cache, scale: float, group=None) -> torch.Tensor:
    """Attention of ``queries`` over a sequence split across the ranks of
    ``group``: this rank's ``cache`` holds its shard (``shard_bounds``), the
    last rank the tail.  Returns the merged output in the query dtype on every
    rank."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    q_len = queries.shape[2]
    if q_len > 1:
        # the chunk's own tokens must all be in the tail shard (it alone is masked); every
        # rank learns the tail's length and all raise together, before any partial exchange
        n = torch.tensor([cache.offset if rank == world - 1 else 0], dtype=torch.int64,
                         device=queries.device if dist.get_backend(group) == "nccl" else "cpu")
        dist.all_reduce(n, op=dist.ReduceOp.MAX, group=group)
        if int(n.item()) < q_len:
            raise ValueError(f"sequence_parallel_attention: the tail shard holds {int(n.item())} tokens, fewer than "
                             f"the {q_len} queries of the chunk; use fewer ranks or a longer sequence")
    o, lse = local_partials(queries, cache, scale, tail=rank == world - 1)
    o_all, lse_all = exchange_partials(o, lse, group)
    return merge_partials(o_all, lse_all, out_dtype=queries.dtype)
