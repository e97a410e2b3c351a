"""ChronoQuant KV cache on B200: paged anchor / residual storage in HBM.

Mirrors ``ChronoQuantCache`` (cache.py:18-287 of the reference): the same
constructor, attributes, cache protocol (``update_and_fetch``, ``offset``,
``make_mask``, ``state``, ``meta_state``, ``is_trimmable``, ``empty``,
``nbytes``) and helper methods, on torch CUDA tensors.

Storage differs from the reference's growing concatenated arrays
(cache.py:118-129): tokens live in fixed-size pages of ``page_tokens`` tokens
(a multiple of lcm(stride_k, stride_v), so every page owns its anchors), each
cut into chunk blocks that hold both components' fp16 anchors, uint32 code
rows and fp16 scales (``PagedStore``).  The anchors and code rows are exactly
the reference's per-token bytes, so ``nbytes`` (the active-byte accounting of
cache.py:274-287) is unchanged; scales are stored per token (2 bytes more per
I-frame).  V code rows use the decode kernel's nibble order when head_dim is
128; ``state`` converts to the reference layout.  ``v_pack=3`` (opt-in, V
codes of 3 bits or fewer) stores V code rows physically in 3 bits per value
(two bit planes, 48 bytes per row at head_dim 128 instead of 64; the decode
kernel reads them for the (64, 32) and (32, 8) stride pairs, the general
kernel otherwise); ``v_pack=2`` (V codes of 2 bits) likewise in one plane of
32 bytes per row.  ``state`` still exports INT4 lanes, and ``nbytes`` keeps
the reference accounting while ``physical_nbytes`` reports what the store
holds.  Appending never copies
history except when the page pool grows (geometrically, or never with
``max_tokens``).
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .trace import traced
from ._tensors import cq_dtype, require_cuda, stream_ptr
from .base import create_causal_mask
from .codec import ChronoQuantCodec

DEFAULT_PAGE_TARGET = 256


def make_causal_mask(offset: int, num_queries: int, return_array: bool = False, window_size=None, device=None):
    """cache.py:7-15: None for one query, "causal" for the implicit rule, or a
    boolean [num_queries, offset] array when asked for (or windowed)."""
    if num_queries == 1:
        return None
    if return_array or (window_size and num_queries > window_size):
        return create_causal_mask(num_queries, offset=offset - num_queries, window_size=window_size, device=device)
    return "causal"


def default_page_tokens(stride_k: int, stride_v: int) -> int:
    """Smallest multiple of lcm(stride_k, stride_v, 16) reaching 256 tokens
    from below (or the lcm itself when larger)."""
    L = math.lcm(int(stride_k), int(stride_v), 16)
    if L >= DEFAULT_PAGE_TARGET:
        return L
    return L * (DEFAULT_PAGE_TARGET // L)


def _num_keyframes(num_tokens: int, stride: int) -> int:
    if num_tokens <= 0:
        return 0
    return ((num_tokens - 1) // stride) + 1


class _Component:
    def __init__(self, stride: int, bits: int, dead_zone: float, page_tokens: int, head_dim: int, order: int):
        self.stride = stride
        # bit-plane rows (head_dim 128): 12 words for 3-bit codes, 8 for 2-bit codes
        self.row_words = {_lib.CQ_ORDER_PLANES3: 12, _lib.CQ_ORDER_PLANES2: 8}.get(order, (head_dim + 7) // 8)
        self.bits = bits
        self.dead_zone = float(dead_zone)
        self.apg = page_tokens // stride
        self.ppg = page_tokens - self.apg
        self.srow = page_tokens  # scales indexed by token position
        self.order = order
        self.off_kf = self.off_cd = self.off_sc = 0  # byte offsets within a chunk block


def _up16(n: int) -> int:
    return (n + 15) & ~15


class PagedStore:
    """Device storage of one cache: one byte buffer of chunk blocks plus the
    block table.

    Pages hold ``P`` tokens, cut into chunks of ``chunk`` tokens (the decode
    kernel's chunk when it takes this configuration, else the whole page).
    Every (page, kv-head, chunk) is one contiguous block

        [K anchors][K code rows][K scales][V anchors][V code rows][V scales]

    (anchors fp16 [chunk/stride][D], code rows uint32 [chunk - chunk/stride]
    [D/8] in P-frame order, scales fp16 [chunk] by token), each segment
    16-byte aligned, so a decode step fetches a chunk with one bulk copy.
    Physical page of (sequence b, logical page p) is ``p * batch + b``; the
    pool grows by reallocating and copying the prefix of pages."""

    def __init__(self, batch: int, heads: int, head_dim: int, page_tokens: int, comps, device):
        self.B, self.H, self.D, self.P = batch, heads, head_dim, page_tokens
        self.W = (head_dim + 7) // 8
        self.comps = comps  # [k, v] _Component
        self.device = device
        c = int(_lib.lib().cq_decode_chunk_tokens(comps[0].stride, comps[1].stride, page_tokens, head_dim))
        self.chunk = c if c > 0 else page_tokens
        off = 0
        for comp in comps:
            a = self.chunk // comp.stride
            comp.off_kf = off
            off = _up16(off + a * head_dim * 2)
            comp.off_cd = off
            off = _up16(off + (self.chunk - a) * comp.row_words * 4)
            comp.off_sc = off
            off = _up16(off + self.chunk * 2)
        self.chunk_bytes = off
        self.head_bytes = (page_tokens // self.chunk) * self.chunk_bytes
        self.max_pages = 0
        self.block_table = None
        self.buf = None
        self._desc = None

    @property
    def n_pages(self) -> int:
        return self.max_pages * self.B

    def capacity_tokens(self) -> int:
        return self.max_pages * self.P

    def ensure(self, tokens: int, hint_tokens: int | None = None) -> None:
        need = max(1, -(-tokens // self.P))
        if need <= self.max_pages:
            return
        target = need
        if hint_tokens:
            target = max(target, -(-int(hint_tokens) // self.P))
        if self.max_pages:
            target = max(target, (self.max_pages * 3 + 1) // 2)
        self._grow(target)

    def _grow(self, max_pages: int) -> None:
        old_n = self.n_pages
        n = max_pages * self.B
        buf = torch.zeros((n, self.H, self.head_bytes), dtype=torch.uint8, device=self.device)
        if old_n:
            buf[:old_n].copy_(self.buf)
        self.buf = buf
        self.max_pages = max_pages
        dev = self.device
        pages = torch.arange(max_pages, dtype=torch.int32, device=dev)
        self.block_table = (pages[None, :] * self.B + torch.arange(self.B, dtype=torch.int32, device=dev)[:, None]
                            ).contiguous()
        self._desc = None

    def descriptor(self) -> _lib.CqPagedCache:
        if self._desc is None:
            d = _lib.CqPagedCache()
            d.batch, d.kv_heads, d.head_dim, d.page_tokens = self.B, self.H, self.D, self.P
            d.max_pages, d.n_pages = self.max_pages, self.n_pages
            d.block_table = self.block_table.data_ptr()
            base = self.buf.data_ptr()
            for name, c in zip(("k", "v"), self.comps):
                cc = getattr(d, name)
                cc.stride, cc.bits, cc.dead_zone = c.stride, c.bits, c.dead_zone
                cc.anchors_per_page, cc.pframes_per_page, cc.scale_row = c.apg, c.ppg, c.srow
                cc.code_order = c.order
                cc.scale_index = _lib.CQ_SCALE_BY_TOKEN
                cc.keyframes, cc.codes, cc.scales = base + c.off_kf, base + c.off_cd, base + c.off_sc
                cc.keyframe_head_stride, cc.code_head_stride = self.head_bytes // 2, self.head_bytes // 4
                cc.scale_head_stride = self.head_bytes // 2
                cc.chunk_tokens = self.chunk
                cc.keyframe_chunk_stride, cc.code_chunk_stride = self.chunk_bytes // 2, self.chunk_bytes // 4
                cc.scale_chunk_stride = self.chunk_bytes // 2
            self._desc = d
        return self._desc

    def pool_bytes(self) -> int:
        return self.buf.numel()


class ChronoQuantCache:
    """ChronoQuant KV cache with paged INT4 residuals and fused attention.

    Arguments follow cache.py:21-31.  Keyword-only extras: ``page_tokens``
    (page size; default the multiple of lcm(stride_k, stride_v, 16) nearest
    256 from below), ``max_tokens`` (pre-size the page pool) and ``v_pack``
    (4: V codes in INT4 lanes as the reference stores them; 3 or 2:
    physically 3 or 2 bits per value, for V codes of at most that many
    bits)."""

    def __init__(self, stride_k: int = 32, stride_v: int = 8, delta_bits_k: int = 4, delta_bits_v: int = 4,
                 dead_zone_k: float = 0.0, dead_zone_v: float = 0.05, use_fused: bool = True,
                 per_layer_v_bits: list = None, layer_idx: int = 0, *, page_tokens: int | None = None,
                 max_tokens: int | None = None, v_pack: int = 4):
        if int(stride_k) < 1 or int(stride_v) < 1:
            raise ValueError("strides must be >= 1")
        self.stride_k = stride_k
        self.stride_v = stride_v
        self.delta_bits_k = delta_bits_k
        self.delta_bits_v = delta_bits_v
        self.dead_zone_k = dead_zone_k
        self.dead_zone_v = dead_zone_v
        self.use_fused = use_fused
        self.per_layer_v_bits = per_layer_v_bits or []
        self.layer_idx = layer_idx
        self.codec_k = ChronoQuantCodec(stride=stride_k, delta_bits=delta_bits_k, dead_zone_ratio=dead_zone_k)
        self.offset = 0
        self.head_dim = None
        if page_tokens is None:
            page_tokens = default_page_tokens(stride_k, stride_v)
        if page_tokens % stride_k or page_tokens % stride_v:
            raise ValueError("page_tokens must be a multiple of stride_k and stride_v")
        self.page_tokens = int(page_tokens)
        self.max_tokens = max_tokens
        if int(v_pack) not in (2, 3, 4):
            raise ValueError("v_pack must be 4 (INT4 lanes), 3 or 2 (physical 3-bit or 2-bit codes)")
        self.v_pack = int(v_pack)
        if self.v_pack < 4:  # (the V codec itself is made lazily: a factory may set layer_idx later)
            v_bits = (self.per_layer_v_bits[min(self.layer_idx, len(self.per_layer_v_bits) - 1)]
                      if self.per_layer_v_bits else self.delta_bits_v)
            if v_bits > self.v_pack:
                raise ValueError(f"v_pack={self.v_pack} needs V codes of at most {self.v_pack} bits, got {v_bits}")
        self._store: PagedStore | None = None
        self._workspace = None

    # -- frame counts (cache.py:53-61) ---------------------------------------
    @staticmethod
    def _num_keyframes(num_tokens: int, stride: int) -> int:
        return _num_keyframes(num_tokens, stride)

    @classmethod
    def _num_pframes(cls, num_tokens: int, stride: int) -> int:
        return num_tokens - cls._num_keyframes(num_tokens, stride)

    # -- storage ----------------------------------------------------------------
    def _get_codec_for_v(self) -> ChronoQuantCodec:
        """cache.py:192-196: V bits from per_layer_v_bits[min(layer_idx, len-1)], else delta_bits_v."""
        if not hasattr(self, "_codec_v") or self._codec_v is None:
            v_bits = (self.per_layer_v_bits[min(self.layer_idx, len(self.per_layer_v_bits) - 1)]
                      if self.per_layer_v_bits else self.delta_bits_v)
            self._codec_v = ChronoQuantCodec(stride=self.stride_v, delta_bits=v_bits, dead_zone_ratio=self.dead_zone_v)
        return self._codec_v

    def _make_store(self, B: int, H: int, D: int, device) -> PagedStore:
        if D % 8 or D > 256:
            raise NotImplementedError(f"head_dim {D} unsupported (multiple of 8, <= 256)")
        cv = self._get_codec_for_v()
        v_order = _lib.CQ_ORDER_MMA if D == 128 else _lib.CQ_ORDER_NATURAL
        if self.v_pack < 4:
            if cv.delta_bits > self.v_pack or D != 128:
                raise ValueError(f"v_pack={self.v_pack} needs V codes of at most {self.v_pack} bits (got "
                                 f"{cv.delta_bits}) and head_dim 128 (got {D})")
            v_order = _lib.CQ_ORDER_PLANES3 if self.v_pack == 3 else _lib.CQ_ORDER_PLANES2
        comps = [_Component(self.stride_k, self.delta_bits_k, self.dead_zone_k, self.page_tokens, D,
                            _lib.CQ_ORDER_NATURAL),
                 _Component(self.stride_v, cv.delta_bits, self.dead_zone_v, self.page_tokens, D, v_order)]
        return PagedStore(B, H, D, self.page_tokens, comps, device)

    @property
    def store(self) -> PagedStore | None:
        return self._store

    # -- cache protocol -----------------------------------------------------------
    @traced("cq.append")
    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        """Encode new K/V tokens into the cache and return the inputs unchanged
        (cache.py:198-215).  keys/values: [B, H_kv, S, head_dim] fp16/bf16 CUDA."""
        if keys.dim() != 4 or values.shape != keys.shape:
            raise ValueError(f"keys/values must be [B, H, S, D] of equal shape, got {tuple(keys.shape)} "
                             f"and {tuple(values.shape)}")
        B, H, S, head_dim = keys.shape
        if self.head_dim is None:
            self.head_dim = head_dim
        elif head_dim != self.head_dim:
            raise ValueError(f"ChronoQuantCache head_dim changed: {self.head_dim} -> {head_dim}")
        require_cuda(keys, values)
        if keys.dtype != values.dtype:
            raise TypeError("keys and values must share a dtype")
        dt = cq_dtype(keys)
        if dt == _lib.CQ_F32:
            raise TypeError("keys/values must be float16 or bfloat16")
        if self._store is None:
            self._store = self._make_store(B, H, head_dim, keys.device)
        elif (B, H) != (self._store.B, self._store.H):
            raise ValueError(f"batch/heads changed: {(self._store.B, self._store.H)} -> {(B, H)}")
        if S == 0:
            return keys, values
        k = keys if keys.stride(-1) == 1 else keys.contiguous()
        v = values if values.stride(-1) == 1 else values.contiguous()
        self._store.ensure(self.offset + S, self.max_tokens)
        d = self._store.descriptor()
        ks, vs = k.stride(), v.stride()
        _lib.check(_lib.lib().cq_append(ctypes.byref(d), k.data_ptr(), ks[0], ks[1], ks[2], v.data_ptr(), vs[0],
                                         vs[1], vs[2], dt, self.offset, S, stream_ptr(k.device)), "update_and_fetch")
        self.offset += S
        return keys, values

    def make_mask(self, num_queries, return_array=False, window_size=None, **kwargs):
        dev = self._store.device if self._store is not None else None
        return make_causal_mask(self.offset, num_queries, return_array, window_size, device=dev)

    def workspace(self, nbytes: int) -> torch.Tensor:
        if self._workspace is None or self._workspace.numel() * 4 < nbytes:
            self._workspace = torch.empty(max(1, (nbytes + 3) // 4), dtype=torch.float32, device=self._store.device)
        return self._workspace

    # -- reference-layout views (cache.py:63-85, 162-190) ---------------------
    def _stride(self, component: str) -> int:
        return self.stride_k if component == "k" else self.stride_v

    def _export(self, component: str):
        """Active (keyframes, packed, scales) of a component in the reference
        layout, materialised from the pages (packed/scales None when the
        component never held a P-frame)."""
        if self._store is None or self.offset == 0:
            return None, None, None
        s = self._stride(component)
        T = self.offset
        nkf = self._num_keyframes(T, s)
        npf = T - nkf
        st = self._store
        dev = st.device
        kf = torch.empty((st.B, st.H, nkf, st.D), dtype=torch.float16, device=dev)
        pk = torch.empty((st.B, st.H, npf, st.W), dtype=torch.uint32, device=dev) if npf else None
        sc = torch.empty((st.B, st.H, npf), dtype=torch.float16, device=dev) if npf else None
        _lib.check(_lib.lib().cq_export_state(ctypes.byref(st.descriptor()), 0 if component == "k" else 1, T,
                                              kf.data_ptr(), None if pk is None else pk.data_ptr(),
                                              None if sc is None else sc.data_ptr(), stream_ptr(dev)), "state")
        return kf, pk, sc

    def _active_keyframes(self, component: str):
        return self._export(component)[0]

    def _active_packed(self, component: str):
        return self._export(component)[1]

    def _active_scales(self, component: str):
        return self._export(component)[2]

    @property
    def keyframes_k(self):
        return self._active_keyframes("k")

    @property
    def keyframes_v(self):
        return self._active_keyframes("v")

    @property
    def packed_codes_k(self):
        return self._active_packed("k")

    @property
    def packed_codes_v(self):
        return self._active_packed("v")

    @property
    def pframe_scales_k(self):
        return self._active_scales("k")

    @property
    def pframe_scales_v(self):
        return self._active_scales("v")

    def _squeezed(self, t):
        if t.shape[0] != 1:
            raise ValueError("kernel_* views are the reference's B=1 views; batch is "
                             f"{t.shape[0]}")
        return t[0]

    def kernel_keyframes_k(self):
        return self._squeezed(self._active_keyframes("k"))

    def kernel_keyframes_v(self):
        return self._squeezed(self._active_keyframes("v"))

    def _zero_placeholder(self, kind: str):
        H, dev = self._store.H, self._store.device
        if kind == "packed":
            return torch.zeros((H, 1, 1), dtype=torch.uint32, device=dev)
        return torch.zeros((H, 1), dtype=torch.float16, device=dev)

    def kernel_packed_k(self):
        p = self._active_packed("k")
        return self._squeezed(p) if p is not None else self._zero_placeholder("packed")

    def kernel_packed_v(self):
        p = self._active_packed("v")
        return self._squeezed(p) if p is not None else self._zero_placeholder("packed")

    def kernel_scales_k(self):
        s = self._active_scales("k")
        return self._squeezed(s) if s is not None else self._zero_placeholder("scales")

    def kernel_scales_v(self):
        s = self._active_scales("v")
        return self._squeezed(s) if s is not None else self._zero_placeholder("scales")

    # -- reconstruction (cache.py:131-160) -----------------------------------
    def _reconstruct_component(self, component: str, mode: int = 0):
        if self.offset == 0 or self._store is None:
            return None
        st = self._store
        out = torch.empty((st.B, st.H, self.offset, st.D), dtype=torch.float16, device=st.device)
        _lib.check(_lib.lib().cq_reconstruct(ctypes.byref(st.descriptor()), 0 if component == "k" else 1,
                                             self.offset, out.data_ptr(), mode, stream_ptr(st.device)),
                   "reconstruct_history")
        return out

    @traced("cq.reconstruct")
    def reconstruct_history(self):
        """Decoded fp16 K and V [B, H, offset, D], rounded as the reference's
        fallback (fp16 code*scale, then fp16 anchor + that)."""
        return self._reconstruct_component("k"), self._reconstruct_component("v")

    # -- state (cache.py:220-272) ------------------------------------------------
    @property
    def state(self):
        if self.offset == 0 or self._store is None:
            return []
        kk, pk, sk = self._export("k")
        kv, pv, sv = self._export("v")
        parts = [kk, kv]
        if pk is not None:
            parts.extend([pk, sk])
        if pv is not None:
            parts.extend([pv, sv])
        return parts

    @state.setter
    def state(self, values):
        """Restore from reference-layout arrays (cache.py:236-255): [kf_k, kf_v,
        (packed_k, scales_k), (packed_v, scales_v)].  offset = K keyframes +
        K P-frames, as the reference computes it."""
        if not values:
            return
        kf_k, kf_v = values[0], values[1]
        packed_k = scales_k = packed_v = scales_v = None
        index = 2
        if len(values) >= 4:
            packed_k, scales_k = values[index], values[index + 1]
            index += 2
        if len(values) >= 6:
            packed_v, scales_v = values[index], values[index + 1]
        require_cuda(kf_k, kf_v)
        B, H, _, D = kf_k.shape
        self.head_dim = D
        T = kf_k.shape[2] + (0 if packed_k is None else packed_k.shape[2])
        self._store = self._make_store(B, H, D, kf_k.device)
        self._store.ensure(T, self.max_tokens)
        self._workspace = None
        d = self._store.descriptor()
        for comp, kf, pk, sc in ((0, kf_k, packed_k, scales_k), (1, kf_v, packed_v, scales_v)):
            s = self.stride_k if comp == 0 else self.stride_v
            nkf = self._num_keyframes(T, s)
            npf = T - nkf
            if kf.shape[2] < nkf or (npf and (pk is None or pk.shape[2] < npf)):
                raise ValueError("state arrays do not cover offset tokens for this cache's strides")
            kfc = kf[:, :, :nkf].to(torch.float16).contiguous()
            pkc = pk[:, :, :npf].contiguous() if npf else None
            scc = sc[:, :, :npf].to(torch.float16).contiguous() if npf else None
            _lib.check(_lib.lib().cq_import_state(ctypes.byref(d), comp, T, kfc.data_ptr(),
                                                  None if pkc is None else pkc.data_ptr(),
                                                  None if scc is None else scc.data_ptr(),
                                                  stream_ptr(kfc.device)), "state")
        self.offset = T

    # The reference's meta_state is "" (cache.py:257-263): a restored cache takes
    # its strides and bits from its constructor.  Here meta_state also carries
    # the configuration, as strings (the prompt-cache file convention), so a
    # saved cache restores self-described; "" is still accepted.
    _META_TAG = "chronoquant/1"
    _META_KEYS = ("stride_k", "stride_v", "delta_bits_k", "delta_bits_v", "dead_zone_k", "dead_zone_v",
                  "use_fused", "per_layer_v_bits", "layer_idx", "page_tokens", "v_pack")

    @property
    def meta_state(self):
        vals = [self.stride_k, self.stride_v, self.delta_bits_k, self.delta_bits_v, repr(float(self.dead_zone_k)),
                repr(float(self.dead_zone_v)), int(bool(self.use_fused)),
                ",".join(str(int(b)) for b in self.per_layer_v_bits), self.layer_idx, self.page_tokens, self.v_pack]
        return (self._META_TAG,) + tuple(f"{k}={v}" for k, v in zip(self._META_KEYS, vals))

    @meta_state.setter
    def meta_state(self, value):
        """Reconfigure an empty cache from ``meta_state`` (set it before
        ``state``).  "" or an empty tuple leaves the configuration as built."""
        if not value:
            return
        if isinstance(value, str):
            value = (value,)
        if value[0] != self._META_TAG:
            raise ValueError(f"unknown meta_state {value[0]!r}")
        if self.offset != 0 or self._store is not None:
            raise ValueError("meta_state can only configure an empty cache")
        kv = dict(item.split("=", 1) for item in value[1:])
        unknown = set(kv) - set(self._META_KEYS)
        if unknown:
            raise ValueError(f"unknown meta_state keys {sorted(unknown)}")
        bits_v = kv.get("per_layer_v_bits", "")
        self.__init__(stride_k=int(kv["stride_k"]), stride_v=int(kv["stride_v"]),
                      delta_bits_k=int(kv["delta_bits_k"]), delta_bits_v=int(kv["delta_bits_v"]),
                      dead_zone_k=float(kv["dead_zone_k"]), dead_zone_v=float(kv["dead_zone_v"]),
                      use_fused=bool(int(kv["use_fused"])),
                      per_layer_v_bits=[int(b) for b in bits_v.split(",")] if bits_v else None,
                      layer_idx=int(kv["layer_idx"]), page_tokens=int(kv["page_tokens"]), max_tokens=self.max_tokens,
                      v_pack=int(kv.get("v_pack", 4)))
        self._codec_v = None  # V bits may have changed

    def is_trimmable(self):
        return False

    def empty(self):
        return self.offset == 0

    def has_previous_state(self) -> bool:
        return self.offset > 0

    # -- active-byte accounting (cache.py:274-287) ------------------------------
    @property
    def nbytes(self) -> int:
        """Sum of the active slices' bytes: fp16 anchors, uint32 code words and
        fp16 scales of K and V (the reference's accounting, not pool size)."""
        if self._store is None or self.offset == 0:
            return 0
        st = self._store
        total = 0
        for s in (self.stride_k, self.stride_v):
            nkf = self._num_keyframes(self.offset, s)
            npf = self.offset - nkf
            total += st.B * st.H * (nkf * st.D * 2 + npf * st.W * 4 + npf * 2)
        return total

    @property
    def physical_nbytes(self) -> int:
        """The same active slices at the bytes the store holds them in: equal to
        ``nbytes`` except with ``v_pack`` 3 or 2, whose V code rows take 3 or 2
        bits per value."""
        if self._store is None or self.offset == 0:
            return 0
        st = self._store
        total = 0
        for s, c in zip((self.stride_k, self.stride_v), st.comps):
            nkf = self._num_keyframes(self.offset, s)
            npf = self.offset - nkf
            total += st.B * st.H * (nkf * st.D * 2 + npf * c.row_words * 4 + npf * 2)
        return total
