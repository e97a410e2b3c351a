"""CPU oracle for the ChronoQuant hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it.  The package ``chronoquant_mlx_b200``
never imports it and has no CPU fallback.

It is a NumPy restatement of the reference's algorithm with the reference's
numeric semantics made explicit:

* every fp16 operation is rounded to fp16 after the operation (MLX computes
  fp16 elementwise ops at fp16 precision; NumPy float16 arithmetic rounds the
  same way: the exact result rounded once to fp16, because fp32/fp64
  intermediates are wide enough for the double rounding to be innocuous);
* Python scalars are weakly typed: ``fp16_array * 0.05`` multiplies by
  ``fp16(0.05)`` and ``fp16_array < 1e-10`` compares against ``fp16(1e-10)``,
  which is 0;
* ``mx.round`` rounds half to even (``np.rint``);
* the float->int8 cast of NaN (an all-zero residual gives 0/0) yields 0, the
  ARM64 ``FCVTZS`` result on the reference's platform.  This is the one
  documented definition where the reference is undefined.

Parity status: pinned.  ``tests/golden/make_golden.py`` runs the reference's
own ``codec.py`` / ``cache.py`` / ``attention.py`` / ``kernels.py`` (unpack)
and its test helpers over a NumPy-backed MLX stand-in and stores the outputs
as fixtures; ``tests/test_oracle_golden.py`` checks this module against them.
MLX's own op semantics (listed above) are assumptions of that stand-in; the
reference's Metal kernels cannot run anywhere here and are restated.

Citations are ``file:line`` in the reference project (gauravsaini/chronoquant_mlx).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F16 = np.float16
F32 = np.float32

# ---------------------------------------------------------------------------
# bf16 emulation (NumPy has no bfloat16): values live in float32 arrays and are
# rounded to the nearest bf16 (ties to even) after every bf16 operation.
# ---------------------------------------------------------------------------


def round_bf16(x) -> np.ndarray:
    """Round float32/float64 values to bf16 precision (RNE), kept as float32."""
    a = np.asarray(x, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    rounded = (bits + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)
    out = rounded.astype(np.uint32).view(np.float32)
    # NaN stays NaN (the add above could carry into the exponent of a NaN)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def bf16_to_bits(x) -> np.ndarray:
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bits_to_bf16(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << np.uint32(16)).view(np.float32)


# ---------------------------------------------------------------------------
# Codec -- codec.py:11-73
# ---------------------------------------------------------------------------


def half_levels(bits: int) -> int:
    """codec.py:14 -- ``(2 ** delta_bits) // 2``."""
    return (2 ** bits) // 2


def _round_to(x64: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return x64.astype(F16)
    if dtype == "bf16":
        return round_bf16(x64.astype(np.float64).astype(np.float32))
    raise ValueError(dtype)


def quantize_delta(delta: np.ndarray, bits: int, dead_zone: float = 0.0, dtype: str = "f16",
                   tie_counter: list | None = None, tie_sites: list | None = None):
    """Restates ``ChronoQuantCodecMLX.quantize_delta`` (codec.py:23-65).

    ``delta``: [..., D] values of the token dtype (fp16, or bf16 held in
    float32).  Every arithmetic step is rounded to that dtype.  Returns
    ``codes`` int8 [..., D] and ``scale`` fp16 [..., 1] (codec.py:65).
    ``tie_counter`` collects the number of quotients exactly halfway between
    two integers (rounded half to even, codec.py:50-51); ``tie_sites`` their
    boolean positions (same shape as ``codes``).
    """
    hl = half_levels(bits)
    d = np.asarray(delta)
    d64 = d.astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        # codec.py:32-33  amax = max|delta|; scale = amax / (hl - 1)
        amax = np.abs(d64).max(axis=-1, keepdims=True)  # exact (max of exact values)
        scale = _round_to(amax / float(hl - 1), dtype).astype(np.float64)
        if dead_zone > 0.0:
            # codec.py:36-45; the weak scalar ratio is rounded to the dtype first
            ratio = float(_round_to(np.float64(dead_zone), dtype))
            thr = _round_to(amax * ratio, dtype).astype(np.float64)
            dz = np.where(np.abs(d64) < thr, 0.0, d64)
            amax_c = np.abs(dz).max(axis=-1, keepdims=True)
            tiny = float(_round_to(np.float64(1e-10), dtype))  # 0 in fp16, 1e-10 in bf16
            amax_safe = np.where(amax_c < tiny, amax, amax_c)
            scale = _round_to(amax_safe / float(hl - 1), dtype).astype(np.float64)
            d64 = dz
        tiny = float(_round_to(np.float64(1e-10), dtype))
        # codec.py:48-54
        scale_safe = np.where(scale < tiny, 1.0, scale)
        q = _round_to(d64 / scale_safe, dtype).astype(np.float64)
        if tie_counter is not None or tie_sites is not None:
            frac = np.abs(q - np.trunc(q))
            if tie_counter is not None:
                tie_counter.append(int(np.count_nonzero(frac == 0.5)))
            if tie_sites is not None:
                tie_sites.append(frac == 0.5)
        r = np.rint(q)
        r = np.clip(r, -hl, hl - 1)
        r = np.where(scale < tiny, 0.0, r)
        r = np.where(np.isnan(r), 0.0, r)  # undefined in the reference; defined as 0 here
    codes = r.astype(np.int8)
    scale_out = scale.astype(F16)  # codec.py:65 scale.astype(float16)
    return codes, scale_out


def dequantize_delta(codes: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """codec.py:67-73: ``codes.astype(f16) * scale`` in fp16."""
    return (codes.astype(F16) * scale.astype(F16)).astype(F16)


# ---------------------------------------------------------------------------
# INT4 packing -- kernels.py:9-61
# ---------------------------------------------------------------------------


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """kernels.py:34-54 (+ the Metal pack kernel kernels.py:9-29).

    nibble = clip(code + 8, 0, 15); word w holds dims 8w..8w+7, dim 8w+i in
    bits 4i..4i+3 (LSB first); the last word is zero-padded.
    """
    c = np.asarray(codes)
    d = c.shape[-1]
    nw = (d + 7) // 8
    nib = np.clip(c.astype(np.int32) + 8, 0, 15).astype(np.uint32)
    if d % 8:
        pad = [(0, 0)] * (nib.ndim - 1) + [(0, nw * 8 - d)]
        nib = np.pad(nib, pad)
    nib = nib.reshape(*c.shape[:-1], nw, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    return np.bitwise_or.reduce(nib << shifts, axis=-1).astype(np.uint32)


def unpack_int4(packed: np.ndarray, head_dim: int) -> np.ndarray:
    """kernels.py:57-61: ``((w >> 4i) & 0xF) - 8`` truncated to ``head_dim``."""
    p = np.asarray(packed, dtype=np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    e = ((p[..., None] >> shifts) & np.uint32(0xF)).astype(np.int32)
    e = e.reshape(*p.shape[:-1], p.shape[-1] * 8)
    return (e[..., :head_dim] - 8).astype(np.int8)


def pack_planes3(codes: np.ndarray) -> np.ndarray:
    """Physical 3-bit rows of this build's opt-in ``v_pack=3`` format (no
    reference counterpart: the reference keeps 3-bit codes in INT4 lanes,
    README.md:57).  ``codes`` int8 [..., 128] in [-4, 3]; v = code + 4 in
    [0, 8).  Returns uint32 [..., 12]: with g = d % 8 and k = d // 8, the low
    two bits of dim d at word g, bit 2k; its high bit at word 8 + g // 2,
    bit 16 (g % 2) + k."""
    c = np.asarray(codes).astype(np.int32)
    assert c.shape[-1] == 128 and c.min(initial=0) >= -4 and c.max(initial=0) <= 3
    v = (c + 4).astype(np.uint32).reshape(*c.shape[:-1], 16, 8)  # [..., k, g]
    k = np.arange(16, dtype=np.uint32)[:, None]
    lo = np.bitwise_or.reduce((v & 3) << (2 * k), axis=-2)  # [..., g]
    hi_g = np.bitwise_or.reduce((v >> 2) << k, axis=-2)     # [..., g]: 16 bits each
    hi = hi_g[..., 0::2] | (hi_g[..., 1::2] << 16)
    return np.concatenate([lo, hi], axis=-1).astype(np.uint32)


def pack_planes2(codes: np.ndarray) -> np.ndarray:
    """Physical 2-bit rows of this build's opt-in ``v_pack=2`` format (no
    reference counterpart).  ``codes`` int8 [..., 128] in [-2, 1]; v = code +
    2 in [0, 4).  Returns uint32 [..., 8]: with g = d % 8 and k = d // 8, dim d
    at word g, bits 2k..2k+1 (the low plane of ``pack_planes3``)."""
    c = np.asarray(codes).astype(np.int32)
    assert c.shape[-1] == 128 and c.min(initial=0) >= -2 and c.max(initial=0) <= 1
    v = (c + 2).astype(np.uint32).reshape(*c.shape[:-1], 16, 8)  # [..., k, g]
    k = np.arange(16, dtype=np.uint32)[:, None]
    return np.bitwise_or.reduce(v << (2 * k), axis=-2).astype(np.uint32)


def unpack_planes2(rows: np.ndarray, head_dim: int = 128) -> np.ndarray:
    """Inverse of ``pack_planes2``: int8 codes [..., 128]."""
    assert head_dim == 128
    r = np.asarray(rows, dtype=np.uint32)
    k = np.arange(16, dtype=np.uint32)[:, None]
    v = (r[..., None, :] >> (2 * k)) & np.uint32(3)  # [..., k, g]
    return (v.astype(np.int32) - 2).reshape(*r.shape[:-1], 128).astype(np.int8)


def unpack_planes3(rows: np.ndarray, head_dim: int = 128) -> np.ndarray:
    """Inverse of ``pack_planes3``: int8 codes [..., 128]."""
    assert head_dim == 128
    r = np.asarray(rows, dtype=np.uint32)
    k = np.arange(16, dtype=np.uint32)[:, None]
    lo = (r[..., None, :8] >> (2 * k)) & np.uint32(3)                       # [..., k, g]
    hi_g = np.stack([r[..., 8:] & np.uint32(0xFFFF), r[..., 8:] >> np.uint32(16)], axis=-1).reshape(
        *r.shape[:-1], 8)
    hi = (hi_g[..., None, :] >> k) & np.uint32(1)
    return ((lo | (hi << 2)).astype(np.int32) - 4).reshape(*r.shape[:-1], 128).astype(np.int8)


# ---------------------------------------------------------------------------
# Frame schedule -- cache.py:53-61, 99-116
# ---------------------------------------------------------------------------


def num_keyframes(n: int, stride: int) -> int:
    """cache.py:53-57."""
    if n <= 0:
        return 0
    return (n - 1) // stride + 1


def num_pframes(n: int, stride: int) -> int:
    """cache.py:59-61."""
    return n - num_keyframes(n, stride)


def active_bytes_per_head(T: int, D: int, stride: int) -> int:
    """Bytes of one component for one (batch, head) row at offset ``T``
    (cache.py:274-287): fp16 anchors + uint32 words + fp16 scales."""
    nkf = num_keyframes(T, stride)
    npf = num_pframes(T, stride)
    return nkf * D * 2 + npf * ((D + 7) // 8) * 4 + npf * 2


def cache_nbytes(B: int, H: int, T: int, D: int, stride_k: int, stride_v: int) -> int:
    """Total active bytes (cache.py:274-287) for K and V."""
    if T <= 0:
        return 0
    return B * H * (active_bytes_per_head(T, D, stride_k) + active_bytes_per_head(T, D, stride_v))


def _to_dtype_array(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return np.asarray(x).astype(F16)
    return round_bf16(np.asarray(x, dtype=np.float32))


def encode_component(x: np.ndarray, t0: int, stride: int, bits: int, dead_zone: float,
                     existing_kf: np.ndarray | None, dtype: str = "f16",
                     tie_counter: list | None = None, tie_sites: list | None = None):
    """Vectorised restatement of ``_append_component`` (cache.py:87-129).

    ``x``: [B, H, S, D] new tokens at absolute positions t0..t0+S-1 (fp16, or
    bf16 values in float32).  ``existing_kf``: fp16 [B, H, n_kf_existing, D].
    Returns the NEW keyframes fp16 [B,H,nk,D], packed uint32 [B,H,np,W] and
    scales fp16 [B,H,np], in token order (cache.py:118-129 concatenates them).
    """
    B, H, S, D = x.shape
    pos = t0 + np.arange(S)
    is_kf = (pos % stride) == 0
    kf_new = np.asarray(x)[:, :, is_kf, :].astype(F16)  # cache.py:103-105 token.astype(f16)
    n_exist = 0 if existing_kf is None else existing_kf.shape[2]
    all_kf = kf_new if existing_kf is None else np.concatenate([existing_kf, kf_new], axis=2)
    pf_pos = pos[~is_kf]
    if pf_pos.size == 0:
        W = (D + 7) // 8
        return kf_new, np.zeros((B, H, 0, W), np.uint32), np.zeros((B, H, 0), F16)
    anchor_idx = pf_pos // stride  # cache.py:107
    assert anchor_idx.max() < all_kf.shape[2], "anchor missing"
    anchors = all_kf[:, :, anchor_idx, :]  # fp16
    tok = np.asarray(x)[:, :, ~is_kf, :]
    # cache.py:113 delta = token - anchor.astype(token.dtype), in the token dtype
    if dtype == "f16":
        delta = (tok.astype(F16).astype(np.float64) - anchors.astype(np.float64)).astype(F16)
    else:
        a_bf = round_bf16(anchors.astype(np.float32))
        delta = round_bf16((tok.astype(np.float64) - a_bf.astype(np.float64)).astype(np.float32))
    codes, scale = quantize_delta(delta, bits, dead_zone, dtype, tie_counter, tie_sites)
    packed = pack_int4(codes)
    return kf_new, packed, scale[..., 0].astype(F16)


def encode_component_loop(x: np.ndarray, t0: int, stride: int, bits: int, dead_zone: float,
                          existing_kf: np.ndarray | None):
    """Reference-structured encode: one token per iteration, as
    ``_append_component``'s loop does (cache.py:99-116).  Used as the
    "reference-structured" CPU baseline; same outputs as ``encode_component``.
    """
    B, H, S, D = x.shape
    kfs, packs, scales = [], [], []
    n_exist = 0 if existing_kf is None else existing_kf.shape[2]
    for lt in range(S):
        t = t0 + lt
        token = x[:, :, lt:lt + 1, :].astype(F16)
        if t % stride == 0:
            kfs.append(token)
            continue
        ai = t // stride
        anchor = existing_kf[:, :, ai:ai + 1, :] if ai < n_exist else kfs[ai - n_exist]
        delta = (token - anchor).astype(F16)
        c, s = quantize_delta(delta, bits, dead_zone)
        packs.append(pack_int4(c))
        scales.append(s[..., 0])
    W = (D + 7) // 8
    kf = np.concatenate(kfs, axis=2) if kfs else np.zeros((B, H, 0, D), F16)
    pk = np.concatenate(packs, axis=2) if packs else np.zeros((B, H, 0, W), np.uint32)
    sc = np.concatenate(scales, axis=2) if scales else np.zeros((B, H, 0), F16)
    return kf, pk, sc


def reconstruct_component(kf: np.ndarray, packed: np.ndarray, scales: np.ndarray, T: int,
                          stride: int, D: int) -> np.ndarray:
    """``_reconstruct_component`` (cache.py:131-156): fp16 anchor gathered per
    position plus the fp16 dequantised delta on P-frames (two fp16 roundings:
    code*scale, then anchor + that)."""
    pos = np.arange(T)
    aidx = pos // stride
    full = kf[:, :, aidx, :].astype(F16)
    if packed is None or packed.shape[2] == 0:
        return full
    pf = np.maximum(pos - aidx - 1, 0)
    is_pf = (pos % stride != 0)[None, None, :, None]
    codes = unpack_int4(packed, D)[:, :, pf, :]
    sc = scales[:, :, pf][..., None]
    delta = dequantize_delta(codes, sc)
    add = np.where(is_pf, delta, F16(0)).astype(F16)
    return (full + add).astype(F16)


def reconstruct_component_f32(kf, packed, scales, T, stride, D) -> np.ndarray:
    """The fused kernel's dequant (kernels.py:152-155, 173-176): fp32
    ``anchor + code * scale`` (computed exactly here, in float64)."""
    pos = np.arange(T)
    aidx = pos // stride
    full = kf[:, :, aidx, :].astype(np.float64)
    if packed is None or packed.shape[2] == 0:
        return full
    pf = np.maximum(pos - aidx - 1, 0)
    is_pf = (pos % stride != 0)[None, None, :, None]
    codes = unpack_int4(packed, D)[:, :, pf, :].astype(np.float64)
    sc = scales[:, :, pf][..., None].astype(np.float64)
    return full + np.where(is_pf, codes * sc, 0.0)


# ---------------------------------------------------------------------------
# Cache -- cache.py:18-287 (reference layout, vectorised append)
# ---------------------------------------------------------------------------


@dataclass
class OracleCache:
    """Restates ``ChronoQuantCache`` (cache.py:18-287) in the reference's own
    storage layout: ``keyframes [B,H,n_kf,D] fp16``, ``packed [B,H,n_pf,W]
    uint32`` and ``scales [B,H,n_pf] fp16`` per component."""

    stride_k: int = 32
    stride_v: int = 8
    delta_bits_k: int = 4
    delta_bits_v: int = 4
    dead_zone_k: float = 0.0
    dead_zone_v: float = 0.05
    per_layer_v_bits: list = field(default_factory=list)
    layer_idx: int = 0
    dtype: str = "f16"
    offset: int = 0
    head_dim: int | None = None
    kf: dict = field(default_factory=dict)
    packed: dict = field(default_factory=dict)
    scales: dict = field(default_factory=dict)

    def v_bits(self) -> int:
        """cache.py:192-196 (lazy V codec bit width)."""
        if self.per_layer_v_bits:
            return self.per_layer_v_bits[min(self.layer_idx, len(self.per_layer_v_bits) - 1)]
        return self.delta_bits_v

    def _append(self, comp, x, stride, bits, dz, tie_counter=None, tie_sites=None):
        kf_new, pk, sc = encode_component(x, self.offset, stride, bits, dz, self.kf.get(comp), self.dtype,
                                          tie_counter, None if tie_sites is None else tie_sites.setdefault(comp, []))
        if kf_new.shape[2]:
            self.kf[comp] = kf_new if comp not in self.kf else np.concatenate([self.kf[comp], kf_new], 2)
        if pk.shape[2]:
            if comp not in self.packed:
                self.packed[comp], self.scales[comp] = pk, sc
            else:
                self.packed[comp] = np.concatenate([self.packed[comp], pk], 2)
                self.scales[comp] = np.concatenate([self.scales[comp], sc], 2)

    def update_and_fetch(self, keys, values, tie_counter=None, tie_sites=None):
        """cache.py:198-215.  ``tie_sites`` (a dict): per component ("k",
        "v") a list of boolean [B, H, n_pframes, D] masks of the halfway
        quotients of each call, in the order of the packed rows."""
        D = keys.shape[-1]
        if self.head_dim is None:
            self.head_dim = D
        elif D != self.head_dim:
            raise ValueError(f"ChronoQuantCache head_dim changed: {self.head_dim} -> {D}")
        self._append("k", keys, self.stride_k, self.delta_bits_k, self.dead_zone_k, tie_counter, tie_sites)
        self._append("v", values, self.stride_v, self.v_bits(), self.dead_zone_v, tie_counter, tie_sites)
        self.offset += keys.shape[2]
        return keys, values

    def stride(self, comp):
        return self.stride_k if comp == "k" else self.stride_v

    def active(self, comp):
        """cache.py:63-85 active slices (keyframes, packed, scales)."""
        s = self.stride(comp)
        nk, npf = num_keyframes(self.offset, s), num_pframes(self.offset, s)
        kf = self.kf.get(comp)
        pk = self.packed.get(comp)
        sc = self.scales.get(comp)
        return (None if kf is None else kf[:, :, :nk],
                None if pk is None else pk[:, :, :npf],
                None if sc is None else sc[:, :, :npf])

    def reconstruct_history(self):
        """cache.py:131-160 (fp16 fallback reconstruction)."""
        out = []
        for comp in ("k", "v"):
            kf, pk, sc = self.active(comp)
            out.append(reconstruct_component(kf, pk, sc, self.offset, self.stride(comp), self.head_dim))
        return tuple(out)

    def reconstruct_history_f32(self):
        out = []
        for comp in ("k", "v"):
            kf, pk, sc = self.active(comp)
            out.append(reconstruct_component_f32(kf, pk, sc, self.offset, self.stride(comp), self.head_dim))
        return tuple(out)

    @property
    def nbytes(self) -> int:
        """cache.py:274-287."""
        total = 0
        for comp in ("k", "v"):
            for a in self.active(comp):
                if a is not None:
                    total += a.size * a.dtype.itemsize
        return total

    @property
    def state(self):
        """cache.py:220-234."""
        if self.offset == 0 or "k" not in self.kf or "v" not in self.kf:
            return []
        kk, pk, sk = self.active("k")
        kv, pv, sv = self.active("v")
        parts = [kk, kv]
        if pk is not None:
            parts += [pk, sk]
        if pv is not None:
            parts += [pv, sv]
        return parts


# ---------------------------------------------------------------------------
# Attention -- attention.py:8-74 and the fused Metal kernel kernels.py:79-228
# ---------------------------------------------------------------------------


def causal_mask(q_len: int, k_len: int) -> np.ndarray:
    """attention.py:13-16: q_idx = arange(Tk-Tq, Tk); mask = q_idx[:,None] >= k_idx."""
    qi = np.arange(k_len - q_len, k_len)
    ki = np.arange(k_len)
    return qi[:, None] >= ki[None]


def _mm(a, b, out_dtype: str):
    """MLX matmul: fp32 accumulation, result rounded to the output dtype."""
    r = np.matmul(a.astype(np.float64), b.astype(np.float64))
    if out_dtype == "f16":
        return r.astype(F16)
    if out_dtype == "bf16":
        return round_bf16(r.astype(np.float32))
    return r.astype(F32)


def _promote(a: str, b: str) -> str:
    """MLX float promotion: fp16 x bf16 -> fp32; same -> same; fp32 wins."""
    if a == b:
        return a
    return "f32"


def fallback_sdpa(queries: np.ndarray, q_dtype: str, full_k: np.ndarray, full_v: np.ndarray,
                  scale: float, mask=None) -> np.ndarray:
    """attention.py:61-74 -- GQA SDPA over the fp16 reconstructed history.

    ``queries``: [B, Hq, Tq, D] (fp16, or bf16 values in float32).
    ``full_k/full_v``: fp16 [B, Hkv, T, D].  Returns the output in the query
    dtype (fp16 array, or bf16 values in float32)."""
    B, Hq, Tq, D = queries.shape
    Hkv = full_k.shape[1]
    rep = Hq // Hkv
    if q_dtype == "f16":
        qs = (queries.astype(np.float64) * float(F16(scale))).astype(F16)
    else:
        qs = round_bf16(queries.astype(np.float64) * float(round_bf16(np.float32(scale))))
    qg = qs.reshape(B, Hkv, rep, Tq, D)
    kg = full_k[:, :, None]
    vg = full_v[:, :, None]
    sdt = _promote(q_dtype, "f16")
    scores = _mm(qg, np.swapaxes(kg, -1, -2), sdt)
    if mask is not None:
        if isinstance(mask, str):
            mask = causal_mask(Tq, full_k.shape[2])
        if mask.dtype == np.bool_:
            fmin = {"f16": -65504.0, "bf16": -3.3895313892515355e38, "f32": float(np.finfo(np.float32).min)}[sdt]
            scores = np.where(mask, scores, fmin)
        else:
            scores = scores + mask
    s64 = scores.astype(np.float64)
    s64 = s64 - s64.max(axis=-1, keepdims=True)
    e = np.exp(s64)
    w = e / e.sum(axis=-1, keepdims=True)
    w = w.astype(F16) if sdt == "f16" else (round_bf16(w.astype(np.float32)) if sdt == "bf16" else w.astype(F32))
    odt = _promote(sdt, "f16")
    out = _mm(w, vg, odt).reshape(B, Hq, Tq, D)
    if q_dtype == "f16":
        return out.astype(np.float64).astype(F16)
    return round_bf16(out.astype(np.float32))


def fused_decode(q_scaled_f32: np.ndarray, kf_k, packed_k, scales_k, kf_v, packed_v, scales_v,
                 T: int, stride_k: int, stride_v: int, D: int) -> np.ndarray:
    """The fused Metal decode kernel (kernels.py:79-228) for B=1, q_len=1,
    evaluated exactly (float64): fp32 dequant ``anchor + code*scale``
    (kernels.py:152-155, 173-176), unscaled dot product (q arrives pre-scaled,
    attention.py:46), softmax over all T tokens, fp32 output [Hq, D].

    ``kf_*``: [Hkv, n_kf, D]; ``packed_*``: [Hkv, n_pf, W]; ``scales_*``:
    [Hkv, n_pf] (the squeezed kernel views, cache.py:162-190)."""
    Hq = q_scaled_f32.shape[0]
    Hkv = kf_k.shape[0]
    rep = Hq // Hkv
    k = reconstruct_component_f32(kf_k[None], packed_k[None], scales_k[None], T, stride_k, D)[0]
    v = reconstruct_component_f32(kf_v[None], packed_v[None], scales_v[None], T, stride_v, D)[0]
    out = np.zeros((Hq, D), np.float64)
    for h in range(Hq):
        kh = h // rep
        s = k[kh] @ q_scaled_f32[h].astype(np.float64)
        s = s - s.max()
        p = np.exp(s)
        out[h] = (p @ v[kh]) / p.sum()
    return out


def exact_sdpa(q_scaled: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool) -> np.ndarray:
    """float64 GQA SDPA on given (already decoded) K/V, q pre-scaled.
    q: [B,Hq,Tq,D]; k,v: [B,Hkv,T,D].  Tie-break reference."""
    B, Hq, Tq, D = q_scaled.shape
    Hkv, T = k.shape[1], k.shape[2]
    rep = Hq // Hkv
    qg = q_scaled.astype(np.float64).reshape(B, Hkv, rep, Tq, D)
    s = np.einsum("bgrqd,bgtd->bgrqt", qg, k.astype(np.float64))
    if causal and Tq > 1:
        m = causal_mask(Tq, T)
        s = np.where(m, s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    o = np.einsum("bgrqt,bgtd->bgrqd", p, v.astype(np.float64)) / p.sum(-1)[..., None]
    return o.reshape(B, Hq, Tq, D)


def lse_merge(ms, ls, os_):
    """Merge partial softmax states (m_i, l_i, o_i) with o_i un-normalised:
    o = sum_i e^{m_i-M} o_i / sum_i e^{m_i-M} l_i."""
    ms = np.asarray(ms, np.float64)
    ls = np.asarray(ls, np.float64)
    os_ = np.asarray(os_, np.float64)
    M = ms.max(axis=0)
    w = np.exp(ms - M)
    num = (w[..., None] * os_).sum(axis=0)
    den = (w * ls).sum(axis=0)
    return num / den[..., None]


# ---------------------------------------------------------------------------
# Synthetic AR(1) KV generator (the measurement spec's workload)
# ---------------------------------------------------------------------------


def ar1_kv(B: int, H: int, T: int, D: int, rho_k: float = 0.95, rho_v: float = 0.8,
           seed: int = 0, n_outliers: int = 4):
    """Per-channel AR(1) keys (innovation sd 0.31, lognormal(0,0.5) channel
    scale, ``n_outliers`` channels x8) and unit-variance AR(1) values, fp16,
    seeded per (b, h) from ``numpy.random.default_rng(seed)``.  Vectorised
    over (b, h); the time recursion is a loop over T."""
    root = np.random.default_rng(seed)
    seeds = root.integers(0, 2**63 - 1, size=(B, H))
    K = np.empty((B, H, T, D), F16)
    V = np.empty((B, H, T, D), F16)
    sd_v = math.sqrt(1.0 - rho_v * rho_v)
    for b in range(B):
        for h in range(H):
            g = np.random.default_rng(int(seeds[b, h]))
            chan = g.lognormal(0.0, 0.5, size=D)
            out_idx = g.choice(D, size=n_outliers, replace=False)
            chan[out_idx] *= 8.0
            ek = g.standard_normal((T, D)) * 0.31
            ev = g.standard_normal((T, D)) * sd_v
            k = np.empty((T, D))
            v = np.empty((T, D))
            k[0] = g.standard_normal(D) * 0.31 / math.sqrt(1 - rho_k * rho_k)
            v[0] = g.standard_normal(D)
            for t in range(1, T):
                k[t] = rho_k * k[t - 1] + ek[t]
                v[t] = rho_v * v[t - 1] + ev[t]
            K[b, h] = (k * chan).astype(F16)
            V[b, h] = v.astype(F16)
    return K, V


def ar1_kv_fast(B: int, H: int, T: int, D: int, rho_k: float = 0.95, rho_v: float = 0.8,
                seed: int = 0, n_outliers: int = 4):
    """Same distribution as ``ar1_kv`` but the recursion runs over all (b, h)
    rows at once (different random stream; used for large benchmark caches)."""
    g = np.random.default_rng(seed)
    chan = g.lognormal(0.0, 0.5, size=(B, H, 1, D)).astype(np.float32)
    for b in range(B):
        for h in range(H):
            idx = g.choice(D, size=n_outliers, replace=False)
            chan[b, h, 0, idx] *= 8.0
    sd_v = math.sqrt(1.0 - rho_v * rho_v)
    K = np.empty((B, H, T, D), F16)
    V = np.empty((B, H, T, D), F16)
    k = (g.standard_normal((B, H, D)) * 0.31 / math.sqrt(1 - rho_k * rho_k)).astype(np.float32)
    v = g.standard_normal((B, H, D)).astype(np.float32)
    chunk = 256
    for t0 in range(0, T, chunk):
        n = min(chunk, T - t0)
        ek = (g.standard_normal((B, H, n, D)) * 0.31).astype(np.float32)
        ev = (g.standard_normal((B, H, n, D)) * sd_v).astype(np.float32)
        for i in range(n):
            if t0 + i > 0:
                k = rho_k * k + ek[:, :, i]
                v = rho_v * v + ev[:, :, i]
            K[:, :, t0 + i] = (k * chan[:, :, 0]).astype(F16)
            V[:, :, t0 + i] = v.astype(F16)
    return K, V
