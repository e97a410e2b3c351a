"""Per-token residual codec on CUDA tensors (codec.py:1-74 of the reference).

``ChronoQuantCodec.quantize_delta`` computes, per (..., token) row over the
head dimension: amax, scale = amax / (half_levels - 1), the optional dead
zone, and codes = clip(round(delta / scale), -half_levels, half_levels - 1),
with every step rounded to the delta's dtype as the reference's MLX fp16/bf16
arithmetic does (codec.py:23-65).  The work runs in ``cq_quantize_delta``.
"""

from __future__ import annotations

import logging

import torch

from . import _lib
from ._tensors import cq_dtype, require_cuda, stream_ptr

log = logging.getLogger("chronoquant_mlx_b200.codec")


class ChronoQuantCodec:
    """Symmetric per-token delta quantisation with optional dead zone.

    Mirrors ``ChronoQuantCodecMLX`` (codec.py:4-21): same constructor
    arguments and attributes.  The reference prints code sparsity every 100
    calls (codec.py:56-63); here that diagnostic is a DEBUG log record, off by
    default, because computing it synchronises the device.
    """

    def __init__(self, stride: int = 32, delta_bits: int = 4, dead_zone_ratio: float = 0.0):
        if not 2 <= int(delta_bits) <= 8:
            raise ValueError(f"delta_bits must be in [2, 8], got {delta_bits}")
        self.stride = stride
        self.delta_bits = delta_bits
        self.half_levels = (2 ** delta_bits) // 2
        self.dead_zone_ratio = dead_zone_ratio
        self._total_elements = 0
        self._zero_elements = 0
        self._log_interval = 100
        self._call_count = 0

    def quantize_delta(self, delta: torch.Tensor):
        """delta [..., head_dim] fp16/bf16 -> (codes int8 [..., head_dim], scale fp16 [..., 1])."""
        require_cuda(delta)
        dt = cq_dtype(delta)
        if dt == _lib.CQ_F32:
            raise TypeError("quantize_delta expects a float16 or bfloat16 residual")
        x = delta.contiguous()
        D = x.shape[-1]
        rows = x.numel() // max(D, 1)
        codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        scales = torch.empty(x.shape[:-1] + (1,), dtype=torch.float16, device=x.device)
        _lib.check(_lib.lib().cq_quantize_delta(x.data_ptr(), dt, rows, D, int(self.delta_bits),
                                                float(self.dead_zone_ratio), codes.data_ptr(), scales.data_ptr(),
                                                stream_ptr(x.device)), "quantize_delta")
        self._call_count += 1
        if self._call_count % self._log_interval == 0 and log.isEnabledFor(logging.DEBUG):
            n_zero = int((codes == 0).sum().item())
            log.debug("[codec] bits=%d dz=%.2f sparsity=%.1f%% (%d/%d zeros)", self.delta_bits,
                      self.dead_zone_ratio, 100.0 * n_zero / max(codes.numel(), 1), n_zero, codes.numel())
        return codes, scales

    def dequantize_delta(self, codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
        """codes.astype(float16) * scale in fp16 (codec.py:67-73); scale [..., 1]."""
        require_cuda(codes, scale)
        c = codes.contiguous()
        D = c.shape[-1]
        rows = c.numel() // max(D, 1)
        s = scale.to(torch.float16).expand(c.shape[:-1] + (1,)).contiguous()
        out = torch.empty(c.shape, dtype=torch.float16, device=c.device)
        _lib.check(_lib.lib().cq_dequantize_delta(c.data_ptr(), s.data_ptr(), rows, D, out.data_ptr(),
                                                  stream_ptr(c.device)), "dequantize_delta")
        return out


# The reference's class name (codec.py:4), for drop-in imports.
ChronoQuantCodecMLX = ChronoQuantCodec
