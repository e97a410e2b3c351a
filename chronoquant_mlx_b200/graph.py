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

``buffers=2`` captures two graphs over two sets of input and output buffers
(they share the cache, its device-resident length and the workspace).  The
sets alternate: ``keys``/``values``/``queries``/``inputs``/``out`` name the
set the next ``replay`` uses, and ``inputs_of(k)`` / ``out_of(k)`` name set
``k % buffers``, so a caller can copy step k+1's inputs in (on another stream)
while step k runs and read step k's output while step k+1 runs.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .trace import traced
from ._tensors import cq_dtype, require_cuda, stream_ptr


class DecodeGraph:
    def __init__(self, cache, num_q_heads: int, scale: float, *, q_dtype=torch.bfloat16, max_len: int | None = None,
                 tokens: int = 1, kv_dtype=torch.float16, out_dtype=None, buffers: int = 1):
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
        if buffers not in (1, 2):
            raise ValueError("buffers must be 1 or 2")
        # a step's inputs live in one flat buffer (one copy fills all three); one set per buffer
        nk = B * H * self.S * D * torch.empty((), dtype=kv_dtype).element_size()
        nq = B * self.Hq * D * torch.empty((), dtype=q_dtype).element_size()
        self._sets = []
        for _ in range(buffers):
            inputs = torch.zeros(2 * nk + nq, dtype=torch.uint8, device=dev)
            self._sets.append(dict(
                inputs=inputs, keys=inputs[:nk].view(kv_dtype).view(B, H, self.S, D),
                values=inputs[nk:2 * nk].view(kv_dtype).view(B, H, self.S, D),
                queries=inputs[2 * nk:].view(q_dtype).view(B, self.Hq, 1, D),
                out=torch.empty((B, self.Hq, 1, D), dtype=out_dtype or q_dtype, device=dev), graph=None))
        self._cur = 0
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
        for i, st_ in enumerate(self._sets):
            self._cur = i
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                if self.S == 1:
                    self._step_fused()  # one kernel: encode each unit's token, then attend
                else:
                    self._append()
                    self._attend()
            st_["graph"] = g
        self._cur = 0
        torch.cuda.synchronize(dev)

    # the buffer set the next replay uses
    @property
    def inputs(self):
        return self._sets[self._cur]["inputs"]

    @property
    def keys(self):
        return self._sets[self._cur]["keys"]

    @property
    def values(self):
        return self._sets[self._cur]["values"]

    @property
    def queries(self):
        return self._sets[self._cur]["queries"]

    @property
    def out(self):
        return self._sets[self._cur]["out"]

    @property
    def graph(self):
        return self._sets[self._cur]["graph"]

    @property
    def buffers(self) -> int:
        return len(self._sets)

    def inputs_of(self, k: int) -> torch.Tensor:
        """Flat input buffer of buffer set ``k % buffers``."""
        return self._sets[k % len(self._sets)]["inputs"]

    def out_of(self, k: int) -> torch.Tensor:
        """Output buffer of buffer set ``k % buffers``."""
        return self._sets[k % len(self._sets)]["out"]

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
        cur = self._sets[self._cur]
        cur["graph"].replay()
        c.offset += self.S
        self._synced = c.offset
        self._cur = (self._cur + 1) % len(self._sets)
        return cur["out"]

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
