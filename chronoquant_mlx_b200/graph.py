"""A decode step captured once as a CUDA graph and replayed every token.

The reference steps eagerly from Python: each token costs an
``update_and_fetch`` (cache.py:198-215) and a ``chronoquant_sdpa``
(attention.py:23-74).  Here the same two operations -- encode the new K/V
token(s) into the paged cache, then attend a one-token query over everything
cached -- run as one CUDA graph whose kernel reads the cache length from
device memory, so the host issues one graph launch per token instead of two
Python-side kernel launches, and the same graph serves every length up to
``max_len``.  With one token per step the graph is a single kernel
(``cq_decode_step_at``: the decode kernel encodes each unit's new token into
the chunk it is about to read); with more, ``cq_append_at`` then
``cq_attention_at``.

Usage::

    g = DecodeGraph(cache, num_q_heads=32, scale=1 / 128 ** 0.5,
                    q_dtype=torch.bfloat16, max_len=T + steps)
    for each token:
        out = g.step(k_new, v_new, q)     # [B, Hq, 1, D], in q_dtype

``step`` copies its inputs into the graph's static buffers (callers may also
write ``g.keys`` / ``g.values`` / ``g.queries`` in place -- views of one flat
byte buffer ``g.inputs``, so a producer can fill all three with one copy --
and call ``replay``),
replays the graph and advances ``cache.offset`` like ``update_and_fetch``.
The returned tensor is the graph's output buffer: it is overwritten by the
next step.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .trace import traced
from ._tensors import cq_dtype, require_cuda, stream_ptr


class DecodeGraph:
    def __init__(self, cache, num_q_heads: int, scale: float, *, q_dtype=torch.bfloat16, max_len: int | None = None,
                 tokens: int = 1, kv_dtype=torch.float16, out_dtype=None):
        st = cache.store
        if st is None or cache.offset == 0:
            raise ValueError("DecodeGraph needs a cache that already holds tokens (prefill first)")
        if not cache.use_fused:
            raise ValueError("DecodeGraph runs the fused decode kernel; this cache has use_fused=False")
        self.cache = cache
        self.S = int(tokens)
        self.max_len = int(max_len) if max_len is not None else st.capacity_tokens()
        if self.max_len < cache.offset + self.S:
            raise ValueError(f"max_len {self.max_len} leaves no room for a step after {cache.offset} tokens")
        st.ensure(self.max_len, cache.max_tokens)  # map every page up front: the graph holds the pointers
        self._buf_ptr = st.buf.data_ptr()
        dev = st.device
        B, H, D = st.B, st.H, st.D
        self.Hq = int(num_q_heads)
        self.scale = float(scale)
        self.len = torch.zeros(2, dtype=torch.int64, device=dev)  # {tokens cached, arrival counter}
        self.len[0] = cache.offset
        self._synced = cache.offset
        # the step's inputs live in one flat buffer (one copy fills all three)
        nk = B * H * self.S * D * torch.empty((), dtype=kv_dtype).element_size()
        nq = B * self.Hq * D * torch.empty((), dtype=q_dtype).element_size()
        self.inputs = torch.zeros(2 * nk + nq, dtype=torch.uint8, device=dev)
        self.keys = self.inputs[:nk].view(kv_dtype).view(B, H, self.S, D)
        self.values = self.inputs[nk:2 * nk].view(kv_dtype).view(B, H, self.S, D)
        self.queries = self.inputs[2 * nk:].view(q_dtype).view(B, self.Hq, 1, D)
        self.out = torch.empty((B, self.Hq, 1, D), dtype=out_dtype or q_dtype, device=dev)
        self._desc = st.descriptor()
        L = _lib.lib()
        need = ctypes.c_size_t(0)
        _lib.check(L.cq_attention_workspace(ctypes.byref(self._desc), self.max_len, self.Hq, 1, 0, ctypes.byref(need)),
                   "DecodeGraph")
        self.workspace = torch.zeros(max(1, (need.value + 3) // 4), dtype=torch.float32, device=dev)
        # one eager attention call (reads only) does the kernels' one-time set-up outside the capture
        torch.cuda.synchronize(dev)
        self._attend()
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            if self.S == 1:
                self._step_fused()  # one kernel: encode each unit's token, then attend
            else:
                self._append()
                self._attend()
        torch.cuda.synchronize(dev)

    def _append(self):
        k, v = self.keys, self.values
        ks, vs = k.stride(), v.stride()
        _lib.check(_lib.lib().cq_append_at(ctypes.byref(self._desc), k.data_ptr(), ks[0], ks[1], ks[2], v.data_ptr(),
                                           vs[0], vs[1], vs[2], cq_dtype(k), self.len.data_ptr(), self.S,
                                           stream_ptr(k.device)), "DecodeGraph")

    def _step_fused(self):
        k, v, q = self.keys, self.values, self.queries
        ks, vs, qs = k.stride(), v.stride(), q.stride()
        _lib.check(_lib.lib().cq_decode_step_at(ctypes.byref(self._desc), k.data_ptr(), ks[0], ks[1], v.data_ptr(),
                                                vs[0], vs[1], cq_dtype(k), self.len.data_ptr(), self.max_len,
                                                q.data_ptr(), cq_dtype(q), self.Hq, qs[0], qs[1], self.scale,
                                                self.out.data_ptr(), cq_dtype(self.out), None,
                                                self.workspace.data_ptr(), self.workspace.numel() * 4,
                                                stream_ptr(q.device)), "DecodeGraph")

    def _attend(self):
        q = self.queries
        qs = q.stride()
        _lib.check(_lib.lib().cq_attention_at(ctypes.byref(self._desc), self.len.data_ptr(), self.max_len,
                                              q.data_ptr(), cq_dtype(q), self.Hq, qs[0], qs[1], self.scale,
                                              self.out.data_ptr(), cq_dtype(self.out), None,
                                              self.workspace.data_ptr(), self.workspace.numel() * 4,
                                              stream_ptr(q.device)), "DecodeGraph")

    @traced("cq.graph_replay")
    def replay(self) -> torch.Tensor:
        """Run one step on the current contents of ``keys``/``values``/``queries``."""
        c = self.cache
        if c.store is None or c.store.buf.data_ptr() != self._buf_ptr:
            raise RuntimeError("the cache's storage moved since capture; build a new DecodeGraph")
        if c.offset != self._synced:  # tokens were appended eagerly in between
            self.len[0] = c.offset
        if c.offset + self.S > self.max_len:
            raise ValueError(f"step past max_len {self.max_len}")
        self.graph.replay()
        c.offset += self.S
        self._synced = c.offset
        return self.out

    @traced("cq.graph_step")
    def step(self, keys: torch.Tensor, values: torch.Tensor, queries: torch.Tensor) -> torch.Tensor:
        """Encode ``keys``/``values`` [B, H, S, D] and attend ``queries``
        [B, Hq, 1, D]; returns the graph's output buffer [B, Hq, 1, D]."""
        require_cuda(keys, values, queries)
        if keys.shape != self.keys.shape or values.shape != self.values.shape or queries.shape != self.queries.shape:
            raise ValueError("step inputs must match the captured shapes")
        self.keys.copy_(keys, non_blocking=True)
        self.values.copy_(values, non_blocking=True)
        self.queries.copy_(queries, non_blocking=True)
        return self.replay()
