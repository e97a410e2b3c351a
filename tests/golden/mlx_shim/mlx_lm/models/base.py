"""Stand-in for ``mlx_lm.models.base``: the attention symbol the reference
patches, and the causal-mask helper its cache imports."""

import mlx.core as mx


CALLS = [0]


def scaled_dot_product_attention(queries, keys, values, cache, scale, mask, **kwargs):
    """Original (un-patched) SDPA symbol; records that it was reached."""
    CALLS[0] += 1
    return "original-sdpa"


def create_causal_mask(N, offset=0, window_size=None):
    rinds = mx.arange(offset + N)
    linds = mx.arange(offset, offset + N)
    mask = linds[:, None] >= rinds[None]
    return mask
