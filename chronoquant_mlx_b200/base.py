"""Host-model side of the plug-in boundary (the role mlx_lm.models.base and
mlx_lm.models.cache play for the reference).

A decoder written against this package calls the module-level
``scaled_dot_product_attention(queries, keys, values, cache, scale, mask)``
and stores keys/values through a cache object with ``update_and_fetch``.
``chronoquant_mlx_b200.apply()`` replaces that symbol so ChronoQuant caches
reach the compressed-cache kernels (patch.py:12-33 of the reference).  The
plain ``KVCache`` and the original SDPA here serve uncompressed layers.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def create_causal_mask(N: int, offset: int = 0, window_size=None, device=None) -> torch.Tensor:
    """Boolean [N, offset + N] mask: query i (absolute offset + i) sees keys
    j <= offset + i, and with a window only keys j > offset + i - window."""
    rinds = torch.arange(offset + N, device=device)
    linds = torch.arange(offset, offset + N, device=device)
    mask = linds[:, None] >= rinds[None]
    if window_size is not None:
        mask = mask & (linds[:, None] < rinds[None] + window_size)
    return mask


def scaled_dot_product_attention(queries, keys, values, cache, scale, mask, **kwargs):
    """Original attention for uncompressed caches (torch SDPA, GQA by repeat)."""
    B, Hq, Tq, D = queries.shape
    Hkv = keys.shape[1]
    if Hq != Hkv:
        keys = keys.repeat_interleave(Hq // Hkv, dim=1)
        values = values.repeat_interleave(Hq // Hkv, dim=1)
    attn_mask, is_causal = None, False
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unknown mask {mask!r}")
        if Tq > 1:
            attn_mask = create_causal_mask(Tq, keys.shape[2] - Tq, device=queries.device)
    elif mask is not None:
        attn_mask = mask
    return F.scaled_dot_product_attention(queries, keys.to(queries.dtype), values.to(queries.dtype),
                                          attn_mask=attn_mask, is_causal=is_causal, scale=scale)


class KVCache:
    """Uncompressed KV cache (the mlx_lm KVCache role): concatenates keys and
    values along the sequence axis."""

    def __init__(self):
        self.keys = None
        self.values = None
        self.offset = 0

    def update_and_fetch(self, keys, values):
        if self.keys is None:
            self.keys, self.values = keys, values
        else:
            self.keys = torch.cat([self.keys, keys], dim=2)
            self.values = torch.cat([self.values, values], dim=2)
        self.offset += keys.shape[2]
        return self.keys, self.values

    def make_mask(self, num_queries, return_array=False, window_size=None, **kwargs):
        if num_queries == 1:
            return None
        if return_array or (window_size and num_queries > window_size):
            return create_causal_mask(num_queries, self.offset - num_queries, window_size,
                                      device=None if self.keys is None else self.keys.device)
        return "causal"

    @property
    def nbytes(self) -> int:
        if self.keys is None:
            return 0
        return self.keys.numel() * self.keys.element_size() + self.values.numel() * self.values.element_size()


def make_prompt_cache(model):
    """One ``KVCache`` per layer (``model.layers``)."""
    return [KVCache() for _ in range(len(model.layers))]
