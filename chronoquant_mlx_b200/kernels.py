"""INT4 packing helpers and the reference-layout fused decode entry
(kernels.py:1-279 of the reference), on CUDA tensors.

The reference's Metal kernels become sm_100a CUDA: ``pack_int4_codes`` and
``unpack_int4_codes`` run ``cq_pack_int4`` / ``cq_unpack_int4``;
``chronoquant_sdpa_kernel`` runs ``cq_sdpa_reference_layout`` on the same
squeezed B=1 views the reference passes (cache.py:162-190).  The cache's own
hot path does not use these: it stores codes in pages and calls
``cq_attention`` (see ``attention.py``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._tensors import require_cuda, stream_ptr

MAX_FUSED_HEAD_DIM = 256  # kernels.py:5


def pack_int4_codes(codes: torch.Tensor) -> torch.Tensor:
    """Pack signed codes into uint32 words: nibble clip(code+8, 0, 15), word w
    holds dims 8w..8w+7 LSB first, last word zero-padded (kernels.py:34-54)."""
    require_cuda(codes)
    c = codes.to(torch.int8).contiguous()
    D = c.shape[-1]
    W = (D + 7) // 8
    rows = c.numel() // max(D, 1)
    out = torch.empty(c.shape[:-1] + (W,), dtype=torch.uint32, device=c.device)
    _lib.check(_lib.lib().cq_pack_int4(c.data_ptr(), rows, D, out.data_ptr(), stream_ptr(c.device)),
               "pack_int4_codes")
    return out


def unpack_int4_codes(packed: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Inverse of ``pack_int4_codes`` truncated to ``head_dim`` (kernels.py:57-61)."""
    require_cuda(packed)
    p = packed.contiguous()
    if p.dtype not in (torch.uint32, torch.int32):
        raise TypeError("packed codes must be uint32 (or int32 holding the same bits)")
    W = p.shape[-1]
    if (head_dim + 7) // 8 != W:
        raise ValueError(f"head_dim {head_dim} does not match {W} packed words")
    rows = p.numel() // max(W, 1)
    out = torch.empty(p.shape[:-1] + (head_dim,), dtype=torch.int8, device=p.device)
    _lib.check(_lib.lib().cq_unpack_int4(p.data_ptr(), rows, head_dim, out.data_ptr(), stream_ptr(p.device)),
               "unpack_int4_codes")
    return out


def chronoquant_sdpa_kernel(q: torch.Tensor, keyframes_k: torch.Tensor, packed_k: torch.Tensor,
                            scales_k: torch.Tensor, keyframes_v: torch.Tensor, packed_v: torch.Tensor,
                            scales_v: torch.Tensor, seq_len: int, stride_k: int, stride_v: int) -> torch.Tensor:
    """Fused decode over reference-layout views for B=1, q_len=1
    (kernels.py:248-279): q fp32 [Hq, D] already scaled; keyframes
    [Hkv, n_kf, D] fp16; packed [Hkv, n_pf, W] uint32; scales [Hkv, n_pf]
    fp16.  Returns fp32 [Hq, D]."""
    require_cuda(q, keyframes_k, packed_k, scales_k, keyframes_v, packed_v, scales_v)
    Hq, D = q.shape
    if D > MAX_FUSED_HEAD_DIM:
        raise ValueError(f"head_dim {D} > {MAX_FUSED_HEAD_DIM}")
    Hkv = keyframes_k.shape[0]
    qf = q.to(torch.float32).contiguous()
    kfk = keyframes_k.to(torch.float16).contiguous()
    kfv = keyframes_v.to(torch.float16).contiguous()
    pk, pv = packed_k.contiguous(), packed_v.contiguous()
    sk = scales_k.to(torch.float16).contiguous()
    sv = scales_v.to(torch.float16).contiguous()
    out = torch.empty((Hq, D), dtype=torch.float32, device=q.device)
    need = ctypes.c_size_t(0)
    _lib.check(_lib.lib().cq_sdpa_reference_layout_workspace(Hq, D, int(seq_len), ctypes.byref(need)),
               "chronoquant_sdpa_kernel")
    ws = torch.empty((need.value + 3) // 4, dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().cq_sdpa_reference_layout(
        qf.data_ptr(), Hq, D, kfk.data_ptr(), kfk.shape[1], pk.data_ptr(), sk.data_ptr(), pk.shape[1],
        kfv.data_ptr(), kfv.shape[1], pv.data_ptr(), sv.data_ptr(), pv.shape[1], Hkv, int(seq_len),
        int(stride_k), int(stride_v), out.data_ptr(), ws.data_ptr(), ws.numel() * 4, stream_ptr(q.device)),
        "chronoquant_sdpa_kernel")
    return out
