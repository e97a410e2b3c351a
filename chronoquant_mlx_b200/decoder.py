"""A random-init Qwen3-style decoder that drives the compressed cache end to
end: greedy decode where every step is one CUDA-graph replay.

Bench config 5 (bench.py --config 5) measures "decode tokens/s at 32k ctx" on a decoder of the
Qwen3-8B shape (36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128,
SwiGLU 12288, vocab 151936, RMSNorm, RoPE theta 1e6, bf16 weights N(0, 0.02))
with Full-Throttle V3 caches.  The reference reaches this through mlx_lm
models calling its patched SDPA (patch.py:12-43); here one module holds the
whole step so that it can be captured:

    per layer: RMSNorm -> fused QKV projection -> per-head q/k RMSNorm -> RoPE
               -> cq_decode_step_at (encode the token into the layer's cache,
                  attend over everything cached: one kernel)
               -> o_proj + residual -> RMSNorm -> SwiGLU FFN + residual
    then: final RMSNorm -> lm_head -> argmax, fed back as the next input ids.

The GEMMs are cuBLAS (torch.matmul); RMSNorm, the per-head q/k norm with
RoPE and the SwiGLU product are this package's fused kernels (cq_rmsnorm,
cq_qk_norm_rope, cq_silu_mul); attention is its decode kernel.  Every layer's cache
length lives on the device and advances inside the kernel, the RoPE position
is a device counter, and the sampled ids are written back in-graph, so a
replay needs no host synchronisation.

Two multi-GPU modes, each inside the captured step, alone or combined on a
mesh of seq x tp ranks (``mesh_groups``): kv-head tensor parallelism
(``tp_group``: NCCL all-reduce after o_proj and the down projection) and a
sequence split of one long context (``seq_group``: each rank's range of
every layer's cache, partial attention with log-sum-exp, one NCCL all-gather
per layer, cq_lse_merge_packed).  Combined, a rank keeps its tensor-parallel
share of the weights and, for its kv-heads, its token range of the context.

``fill_context`` writes a synthetic context (seeded random K/V per layer,
encoded by the cache's own append kernel) instead of running a 32k-token
prompt through the model; a decode step's cost does not depend on the
values.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._tensors import cq_dtype, stream_ptr
from .cache import ChronoQuantCache


@dataclass
class DecoderConfig:
    layers: int = 36
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 12288
    vocab: int = 151936
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6


def mesh_groups(seq: int, tp: int):
    """Process groups of a seq x tp mesh over the default group's ranks
    r = s * tp + p (seq index s, tensor-parallel index p): the tensor-parallel
    group of this rank (ranks with its s) and its sequence group (ranks with
    its p).  Every rank creates every group, in the same order, as
    torch.distributed requires.  Returns (tp_group, seq_group); a size-1
    dimension gives None."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(), dist.get_rank()
    if seq < 1 or tp < 1 or seq * tp != world:
        raise ValueError(f"mesh {seq} x {tp} does not cover the {world} ranks")
    tp_group = seq_group = None
    for s in range(seq):
        g = dist.new_group([s * tp + p for p in range(tp)])
        if rank // tp == s:
            tp_group = g
    for p in range(tp):
        g = dist.new_group([s * tp + p for s in range(seq)])
        if rank % tp == p:
            seq_group = g
    return (tp_group if tp > 1 else None), (seq_group if seq > 1 else None)


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm as the torch expression that cq_rmsnorm reproduces (the tests'
    reference for the fused kernel)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of x [B, H, D] at one position (cos/sin [D])."""
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), dim=-1)
    return (x.float() * cos + rot.float() * sin).to(x.dtype)


class Qwen3StyleDecoder:
    """Random-init weights, one ChronoQuantCache per layer, and a graph-captured
    greedy decode step for ``batch`` sequences of up to ``max_len`` tokens."""

    def __init__(self, cfg: DecoderConfig, batch: int, max_len: int, cache_kwargs: dict | None = None,
                 device="cuda", dtype=torch.bfloat16, seed: int = 0, tp_group=None, seq_group=None,
                 peer_sum: bool = True):
        """``tp_group``: a torch.distributed (NCCL) group over which the layers
        are tensor-parallel by kv-head: this rank keeps kv_heads/N kv-heads
        with their query heads and ffn/N of each FFN; the o_proj and down
        projections end in an all-reduce.  The full weights are drawn the same
        way on every rank and sliced, so any N gives the same model.

        ``seq_group``: a group over which every sequence's context is split
        by token ranges (``distributed.shard_bounds``): each rank keeps the
        whole model and, per layer, the compressed cache of its range; the
        last rank owns the tail and encodes the new tokens.  Each layer's
        attention is a partial (output, log-sum-exp) per rank, all-gathered
        (NCCL) and merged by cq_lse_merge_packed, all inside the captured step.

        ``peer_sum`` (tensor parallel): each row-parallel projection's sum
        over the ranks, with the residual add and the next RMSNorm, is one
        ``PeerSumNorm`` kernel reading the other ranks' parts over NVLink;
        False uses an NCCL all-reduce followed by the separate add and norm.

        Both together (``mesh_groups``): the layers are tensor-parallel over
        ``tp_group`` and each rank's kv-heads hold its token range of the
        context; the tail ranks (the last of every sequence group) encode the
        new tokens."""
        self.cfg, self.B, self.max_len = cfg, batch, max_len
        self.device, self.dtype = torch.device(device), dtype
        self.group, self.seq_group = tp_group, seq_group
        self.seq_rank, self.seq_world = 0, 1
        if seq_group is not None:
            import torch.distributed as dist
            self.seq_rank, self.seq_world = dist.get_rank(seq_group), dist.get_world_size(seq_group)
        self.tail = self.seq_rank == self.seq_world - 1  # this rank encodes the new tokens
        if tp_group is not None:
            import torch.distributed as dist
            self.rank, self.world = dist.get_rank(tp_group), dist.get_world_size(tp_group)
        else:
            self.rank, self.world = 0, 1
        c = cfg
        if c.kv_heads % self.world or c.ffn % self.world:
            raise ValueError("kv_heads and ffn must divide by the tensor-parallel size")
        self.heads, self.kv_heads, self.ffn = c.heads // self.world, c.kv_heads // self.world, c.ffn // self.world
        g = torch.Generator(device=self.device).manual_seed(seed)

        def w(*shape):
            return (torch.randn(shape, generator=g, device=self.device, dtype=torch.float32) * 0.02).to(dtype)

        r, D = self.rank, c.head_dim
        hq, hk, f = self.heads, self.kv_heads, self.ffn

        def local_qkv(full):  # rows [q heads | k heads | v heads] -> this rank's heads of each
            q0, k0 = c.heads * D, (c.heads + c.kv_heads) * D
            return torch.cat((full[r * hq * D:(r + 1) * hq * D], full[q0 + r * hk * D:q0 + (r + 1) * hk * D],
                              full[k0 + r * hk * D:k0 + (r + 1) * hk * D])).contiguous()

        self.embed = w(c.vocab, c.hidden)
        self.lm_head = w(c.vocab, c.hidden)
        self.final_norm = torch.ones(c.hidden, device=self.device, dtype=dtype)
        self.layers = []
        for i in range(c.layers):
            wqkv = local_qkv(w((c.heads + 2 * c.kv_heads) * D, c.hidden))
            wo = w(c.hidden, c.heads * D)[:, r * hq * D:(r + 1) * hq * D].contiguous()
            wgu_full = w(2 * c.ffn, c.hidden)
            wgu = torch.cat((wgu_full[r * f:(r + 1) * f], wgu_full[c.ffn + r * f:c.ffn + (r + 1) * f])).contiguous()
            del wgu_full
            wdown = w(c.hidden, c.ffn)[:, r * f:(r + 1) * f].contiguous()
            self.layers.append(dict(
                ln1=torch.ones(c.hidden, device=self.device, dtype=dtype),
                ln2=torch.ones(c.hidden, device=self.device, dtype=dtype),
                q_norm=torch.ones(D, device=self.device, dtype=dtype),
                k_norm=torch.ones(D, device=self.device, dtype=dtype),
                wqkv=wqkv, wo=wo, wgu=wgu, wdown=wdown,
                cache=ChronoQuantCache(layer_idx=i, max_tokens=max_len, **(cache_kwargs or {})),
            ))
        self.inv_freq = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=self.device,
                                                             dtype=torch.float32) / c.head_dim))
        self.ids = torch.zeros(batch, dtype=torch.long, device=self.device)  # input ids of the next step
        self.pos = torch.zeros((), dtype=torch.long, device=self.device)   # their position
        self.out_ids = torch.zeros(batch, dtype=torch.long, device=self.device)
        self.graph = None
        self.peer = None
        if self.world > 1 and peer_sum:
            from .peer import PeerSumNorm
            self.peer = PeerSumNorm(tp_group, batch, c.hidden, device=self.device)

    # -- context ---------------------------------------------------------------
    def fill_context(self, T0: int, chunk: int = 4096, seed: int = 1) -> None:
        """Encode a synthetic T0-token context into every layer's cache (under
        a sequence split, this rank's token range of it)."""
        c = self.cfg
        g = torch.Generator(device=self.device).manual_seed(seed)
        h0, h1 = self.rank * self.kv_heads, (self.rank + 1) * self.kv_heads  # this rank's kv-heads
        t_lo, t_hi = 0, T0
        if self.seq_group is not None:
            from .distributed import shard_bounds
            c0 = self.layers[0]["cache"]
            t_lo, t_hi = shard_bounds(T0, self.seq_world, c0.stride_k, c0.stride_v)[self.seq_rank]
            if t_hi <= t_lo:
                raise ValueError("sequence split: every rank needs a non-empty token range")
        for L in self.layers:
            for t in range(0, T0, chunk):
                n = min(chunk, T0 - t)
                k = torch.randn((self.B, c.kv_heads, n, c.head_dim), generator=g, device=self.device).to(self.dtype)
                v = torch.randn((self.B, c.kv_heads, n, c.head_dim), generator=g, device=self.device).to(self.dtype)
                a, b = max(t, t_lo) - t, min(t + n, t_hi) - t  # the part of this chunk in the rank's range
                if a < b:
                    L["cache"].update_and_fetch(k[:, h0:h1, a:b].contiguous(), v[:, h0:h1, a:b].contiguous())
        self.pos.fill_(T0)
        self._prepare_attention()

    def _prepare_attention(self) -> None:
        """Per-layer descriptors, device-resident lengths and one shared
        workspace (layers run in order on one stream)."""
        lib = _lib.lib()
        need_max = 0
        for L in self.layers:
            st = L["cache"].store
            st.ensure(self.max_len, self.max_len)
            L["desc"] = st.descriptor()
            L["len"] = torch.tensor([L["cache"].offset, 0], dtype=torch.int64, device=self.device)
            need = ctypes.c_size_t(0)
            _lib.check(lib.cq_attention_workspace(ctypes.byref(L["desc"]), self.max_len, self.heads, 1, 0,
                                                  ctypes.byref(need)), "decoder")
            need_max = max(need_max, need.value)
        self.workspace = torch.zeros(max(1, (need_max + 3) // 4), dtype=torch.float32, device=self.device)
        self.attn_out = torch.empty((self.B, self.heads, self.cfg.head_dim), dtype=self.dtype, device=self.device)
        if self.seq_group is not None:
            # this rank's partial packed as [outputs B*Hq*D | log-sum-exp B*Hq] (one all-gather per
            # layer), and every rank's, gathered rank-major
            W, D, R = self.seq_world, self.cfg.head_dim, self.B * self.heads
            self.part = torch.empty(R * (D + 1), dtype=torch.float32, device=self.device)
            self.o_part = self.part[:R * D].view(self.B, self.heads, D)
            self.lse_part = self.part[R * D:].view(self.B, self.heads)
            self.parts_all = torch.empty((W, R * (D + 1)), dtype=torch.float32, device=self.device)

    # -- one decode step --------------------------------------------------------
    def _attention(self, L: dict, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Encode this step's k/v [B, Hkv, D] into the layer's cache and attend
        q [B, Hq, D] over everything cached: one cq_decode_step_at launch.
        Under a sequence split the tail rank does that and the others attend
        their fixed range (cq_attention_at); each writes an fp32 partial with
        its log-sum-exp, and the gathered partials are merged (cq_lse_merge_packed)."""
        lib = _lib.lib()
        ks, vs, qs = k.stride(), v.stride(), q.stride()
        scale = 1.0 / math.sqrt(self.cfg.head_dim)
        split = self.seq_group is not None
        out = self.o_part if split else self.attn_out
        lse = self.lse_part.data_ptr() if split else None
        if self.tail:
            _lib.check(lib.cq_decode_step_at(
                ctypes.byref(L["desc"]), k.data_ptr(), ks[0], ks[1], v.data_ptr(), vs[0], vs[1], cq_dtype(k),
                L["len"].data_ptr(), self.max_len, q.data_ptr(), cq_dtype(q), self.heads, qs[0], qs[1], scale,
                out.data_ptr(), cq_dtype(out), lse, self.workspace.data_ptr(), self.workspace.numel() * 4,
                stream_ptr(self.device)), "decoder")
        else:
            _lib.check(lib.cq_attention_at(
                ctypes.byref(L["desc"]), L["len"].data_ptr(), self.max_len, q.data_ptr(), cq_dtype(q), self.heads,
                qs[0], qs[1], scale, out.data_ptr(), cq_dtype(out), lse, self.workspace.data_ptr(),
                self.workspace.numel() * 4, stream_ptr(self.device)), "decoder")
        if split:
            self._merge_partials()
        return self.attn_out

    def _gather_partials(self) -> None:
        """Every rank's packed partial into parts_all (rank-major)."""
        import torch.distributed as dist
        dist.all_gather_into_tensor(self.parts_all, self.part, group=self.seq_group)

    def _merge_partials(self) -> None:
        self._gather_partials()
        _lib.check(_lib.lib().cq_lse_merge_packed(self.parts_all.data_ptr(), self.seq_world, self.B * self.heads,
                                                  self.cfg.head_dim, self.attn_out.data_ptr(),
                                                  cq_dtype(self.attn_out), stream_ptr(self.device)), "decoder")

    def _norm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        y = torch.empty_like(x)
        _lib.check(_lib.lib().cq_rmsnorm(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1],
                                         self.cfg.eps, cq_dtype(x), stream_ptr(self.device)), "decoder")
        return y

    def _reduce(self, partial: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel projection's partial outputs over the tensor-parallel ranks."""
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(partial, group=self.group)
        return partial

    def _project_sum_norm(self, x: torch.Tensor, a: torch.Tensor, wt: torch.Tensor, w_norm: torch.Tensor,
                          parity: int) -> torch.Tensor:
        """x <- x + (sum over the tensor-parallel ranks of a @ wt.T); returns
        RMSNorm(x) * w_norm.  With peer sums one kernel pushes this rank's part
        to every rank and does the sum, the add and the norm."""
        if self.peer is not None:
            y = torch.empty_like(x)
            self.peer(a @ wt.t(), x, w_norm, self.cfg.eps, y, parity)
            return y
        x += self._reduce(a @ wt.t())
        return self._norm(x, w_norm)

    def _step_body(self, attention=None) -> torch.Tensor:
        c, B = self.cfg, self.B
        attention = attention or self._attention
        nq, nk = self.heads * c.head_dim, self.kv_heads * c.head_dim
        lib, st, dt = _lib.lib(), stream_ptr(self.device), cq_dtype(self.embed)
        x = self.embed[self.ids]  # a fresh tensor: updated in place below
        xn = self._norm(x, self.layers[0]["ln1"])
        parity = 0  # peer part buffers alternate per call; a step makes an even number of calls
        for i, L in enumerate(self.layers):
            qkv = xn @ L["wqkv"].t()
            q = torch.empty((B, self.heads, c.head_dim), device=self.device, dtype=self.dtype)
            k = torch.empty((B, self.kv_heads, c.head_dim), device=self.device, dtype=self.dtype)
            v = torch.empty_like(k)
            _lib.check(lib.cq_qk_norm_rope(qkv.data_ptr(), qkv.stride(0), B, self.heads, self.kv_heads, c.head_dim,
                                           L["q_norm"].data_ptr(), L["k_norm"].data_ptr(), self.inv_freq.data_ptr(),
                                           self.pos.data_ptr(), c.eps, q.data_ptr(), k.data_ptr(), v.data_ptr(), dt,
                                           st), "decoder")
            a = attention(L, q, k, v)
            xn = self._project_sum_norm(x, a.reshape(B, nq), L["wo"], L["ln2"], parity)
            parity ^= 1
            gu = xn @ L["wgu"].t()
            h = torch.empty((B, self.ffn), device=self.device, dtype=self.dtype)
            _lib.check(lib.cq_silu_mul(gu.data_ptr(), h.data_ptr(), B, self.ffn, dt, st), "decoder")
            w_next = self.layers[i + 1]["ln1"] if i + 1 < len(self.layers) else self.final_norm
            xn = self._project_sum_norm(x, h, L["wdown"], w_next, parity)
            parity ^= 1
        logits = xn @ self.lm_head.t()
        self.out_ids.copy_(logits.argmax(-1))
        self.ids.copy_(self.out_ids)
        self.pos.add_(1)
        return logits

    def step_eager(self, attention=None) -> torch.Tensor:
        """One decode step without a graph (``attention(L, q, k, v)`` may
        replace the kernel, e.g. by a reference).  Returns logits [B, vocab]."""
        return self._step_body(attention)

    def capture(self) -> None:
        """Capture one decode step as a CUDA graph (after ``fill_context``)."""
        lib = _lib.lib()
        c = self.cfg
        # one-time set-up outside the capture: cuBLAS handles (one matmul of each
        # shape) and the attention kernel's attributes (a read-only attention call)
        x = torch.zeros((self.B, c.hidden), device=self.device, dtype=self.dtype)
        L0 = self.layers[0]
        for wt in (L0["wqkv"], L0["wgu"], self.lm_head):
            x @ wt.t()
        (torch.zeros((self.B, self.ffn), device=self.device, dtype=self.dtype) @ L0["wdown"].t())
        if self.world > 1 and self.peer is None:  # the communicator exists before the capture
            self._reduce(torch.zeros((self.B, c.hidden), device=self.device, dtype=self.dtype))
        if self.seq_group is not None:
            self.o_part.zero_()
            self.lse_part.zero_()
            self._merge_partials()
        q = torch.zeros((self.B, self.heads, c.head_dim), device=self.device, dtype=self.dtype)
        qs = q.stride()
        _lib.check(lib.cq_attention_at(ctypes.byref(L0["desc"]), L0["len"].data_ptr(), self.max_len, q.data_ptr(),
                                       cq_dtype(q), self.heads, qs[0], qs[1], 1.0, self.attn_out.data_ptr(),
                                       cq_dtype(self.attn_out), None, self.workspace.data_ptr(),
                                       self.workspace.numel() * 4, stream_ptr(self.device)), "decoder")
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._step_body()
        torch.cuda.synchronize(self.device)

    def decode(self, steps: int) -> torch.Tensor:
        """Replay the captured step ``steps`` times (greedy, no host sync in
        between); returns the last step's logits.  The caches' host-side
        offsets follow the device lengths afterwards."""
        start = self.layers[0]["cache"].offset
        if start + steps > self.max_len:
            raise ValueError(f"decode past max_len {self.max_len}")
        for _ in range(steps):
            self.graph.replay()
        if self.tail:  # under a sequence split only the tail rank's caches grow
            for L in self.layers:
                L["cache"].offset += steps
        return self.logits

    def close(self) -> None:
        """Release the peer-memory regions (collective over the tensor-parallel
        group; after the graphs are gone, before the process group)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def bytes_per_step(self) -> int:
        """Algorithmic HBM bytes of one step: every weight once, every layer's
        active compressed cache once (the reference accounting)."""
        w = self.embed.shape[1] * self.embed.element_size() * self.B + self.lm_head.numel() * self.lm_head.element_size()
        for L in self.layers:
            w += sum(L[n].numel() * L[n].element_size() for n in ("wqkv", "wo", "wgu", "wdown"))
            w += L["cache"].nbytes
        return w
