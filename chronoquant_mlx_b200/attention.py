"""ChronoQuant attention dispatch on B200 (attention.py:1-74 of the reference).

The reference runs its fused Metal kernel only for B=1, q_len=1 and otherwise
reconstructs the whole fp16 history and calls generic matmul/softmax
(attention.py:34-74).  Here every case runs on the GPU through the C ABI:

* ``use_fused`` and mask None/"causal": ``cq_attention`` reads the paged
  compressed cache directly, for any batch and any q_len (decode is the
  split-KV kernel; longer query chunks use the causal rule anchored at the
  end of the keys, attention.py:8-20);
* an explicit array mask: ``cq_attention_masked`` (boolean masks fill
  finfo(score dtype).min, additive masks add, as attention.py:17-20);
* ``use_fused=False``: the reference's fallback order -- decode the fp16
  history (``cq_reconstruct``, its fp16 rounding) and attend over it with the
  same kernels.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .trace import traced
from ._tensors import cq_dtype, require_cuda, stream_ptr


def _dense_descriptor(k: torch.Tensor, v: torch.Tensor, table: torch.Tensor) -> _lib.CqPagedCache:
    """Descriptor of plain fp16 [B, H, T, D] K/V as a stride-1 cache (every
    token an I-frame, one page per sequence)."""
    B, H, T, D = k.shape
    d = _lib.CqPagedCache()
    d.batch, d.kv_heads, d.head_dim, d.page_tokens = B, H, D, T
    d.max_pages, d.n_pages = 1, B
    d.block_table = table.data_ptr()
    for name, t in (("k", k), ("v", v)):
        c = getattr(d, name)
        c.stride, c.bits, c.dead_zone = 1, 4, 0.0
        c.anchors_per_page, c.pframes_per_page, c.scale_row = T, 0, 0
        c.code_order = _lib.CQ_ORDER_NATURAL
        c.scale_index = _lib.CQ_SCALE_BY_PFRAME
        c.keyframes, c.codes, c.scales = t.data_ptr(), None, None
    return d


def _mask_args(mask: torch.Tensor, B: int, Hq: int, Tq: int, T: int):
    m = mask
    if m.dim() > 4:
        raise ValueError("mask must have at most 4 dims [B, H, Tq, T]")
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.shape[-1] != T or m.shape[-2] not in (1, Tq):
        raise ValueError(f"mask shape {tuple(mask.shape)} does not broadcast to [{B}, {Hq}, {Tq}, {T}]")
    if m.dtype == torch.bool:
        m = m.to(torch.uint8)
        kind, mdt = 1, _lib.CQ_F32
    else:
        kind, mdt = 2, cq_dtype(m)
    strides = [0 if m.shape[i] == 1 else m.stride(i) for i in range(4)]
    return m, kind, mdt, strides


def _run(desc, T, queries, scale, mask, causal, out, ws_holder, device):
    B, Hq, Tq, D = queries.shape
    q = queries if queries.stride(-1) == 1 else queries.contiguous()
    qs = q.stride()
    L = _lib.lib()
    need = ctypes.c_size_t(0)
    _lib.check(L.cq_attention_workspace(ctypes.byref(desc), T, Hq, Tq, 0, ctypes.byref(need)), "chronoquant_sdpa")
    ws = ws_holder(need.value)
    qdt = cq_dtype(q)
    odt = cq_dtype(out)
    if mask is None or isinstance(mask, str):
        _lib.check(L.cq_attention(ctypes.byref(desc), T, q.data_ptr(), qdt, Hq, Tq, 1 if causal else 0, qs[0],
                                  qs[1], qs[2], float(scale), out.data_ptr(), odt, None, ws.data_ptr(),
                                  ws.numel() * 4, 0, stream_ptr(device)), "chronoquant_sdpa")
    else:
        require_cuda(mask)
        m, kind, mdt, ms = _mask_args(mask, B, Hq, Tq, T)
        _lib.check(L.cq_attention_masked(ctypes.byref(desc), T, q.data_ptr(), qdt, Hq, Tq, qs[0], qs[1], qs[2],
                                         float(scale), m.data_ptr(), kind, mdt, ms[0], ms[1], ms[2], ms[3],
                                         out.data_ptr(), odt, ws.data_ptr(), ws.numel() * 4, 0,
                                         stream_ptr(device)), "chronoquant_sdpa")
    return out


@traced("cq.sdpa")
def chronoquant_sdpa(queries: torch.Tensor, keys, values, cache, scale: float, mask=None):
    """Attention of ``queries`` [B, Hq, Tq, D] (fp16/bf16 CUDA) over everything
    ``cache`` holds, including tokens just appended by ``update_and_fetch``.
    ``keys``/``values`` are the placeholders the cache returned and are not
    read (attention.py:23-30).  Returns [B, Hq, Tq, D] in the query dtype."""
    B, Hq, Tq, D = queries.shape
    require_cuda(queries)
    if cache.offset == 0 or cache.store is None:
        raise ValueError("chronoquant_sdpa: the cache is empty")
    if isinstance(mask, str) and mask != "causal":
        raise ValueError(f"unknown mask {mask!r}")
    st = cache.store
    if D != st.D:
        raise ValueError(f"query head_dim {D} != cache head_dim {st.D}")
    T = cache.offset
    out = torch.empty((B, Hq, Tq, D), dtype=queries.dtype, device=queries.device)
    causal = isinstance(mask, str)
    if cache.use_fused:
        return _run(st.descriptor(), T, queries, scale, mask, causal, out, cache.workspace, queries.device)
    full_k, full_v = cache.reconstruct_history()
    table = torch.arange(B, dtype=torch.int32, device=queries.device)
    desc = _dense_descriptor(full_k, full_v, table)
    return _run(desc, T, queries, scale, mask, causal, out, cache.workspace, queries.device)


@traced("cq.sdpa_lse")
def chronoquant_sdpa_with_lse(queries: torch.Tensor, cache, scale: float, causal: bool = True):
    """Decode/prefill attention returning (out fp32 [B, Hq, Tq, D], lse fp32
    [B, Hq, Tq]) for merging sequence shards (``distributed.py``).  ``causal``
    applies the end-anchored causal mask when Tq > 1 (no effect for Tq 1); a
    shard whose keys all precede the queries passes False."""
    B, Hq, Tq, D = queries.shape
    require_cuda(queries)
    st = cache.store
    T = cache.offset
    out = torch.empty((B, Hq, Tq, D), dtype=torch.float32, device=queries.device)
    lse = torch.empty((B, Hq, Tq), dtype=torch.float32, device=queries.device)
    q = queries if queries.stride(-1) == 1 else queries.contiguous()
    qs = q.stride()
    desc = st.descriptor()
    L = _lib.lib()
    need = ctypes.c_size_t(0)
    _lib.check(L.cq_attention_workspace(ctypes.byref(desc), T, Hq, Tq, 0, ctypes.byref(need)), "attention")
    ws = cache.workspace(need.value)
    _lib.check(L.cq_attention(ctypes.byref(desc), T, q.data_ptr(), cq_dtype(q), Hq, Tq, 1 if causal else 0, qs[0],
                              qs[1], qs[2], float(scale), out.data_ptr(), _lib.CQ_F32, lse.data_ptr(), ws.data_ptr(),
                              ws.numel() * 4, 0, stream_ptr(queries.device)), "attention")
    return out, lse
