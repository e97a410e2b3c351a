"""Hugging Face ``transformers`` integration: ChronoQuant caches and attention
for transformers models (real checkpoints) on the B200 kernels.

The reference plugs into mlx_lm by replacing its SDPA symbol and dispatching
on the cache type (patch.py:12-43); the cache keeps the KV and the SDPA reads
it (cache.py:198-215, attention.py:23-74).  transformers has the same two
seams: a registry of attention functions selected by
``config._attn_implementation`` (``AttentionInterface``), and a cache
protocol (``Cache`` made of per-layer ``CacheLayerMixin``).  This module
fills both:

* ``ChronoQuantHFCache`` -- a ``Cache`` whose layer i is a
  ``ChronoQuantCache(layer_idx=i, **kwargs)``.  ``update`` encodes the new
  K/V tokens into the compressed store and, like the reference's
  ``update_and_fetch``, returns the inputs unchanged, tagged with their cache;
* ``chronoquant_attention`` -- registered as ``"chronoquant"``: for keys
  tagged by a ChronoQuant layer it runs ``chronoquant_sdpa`` over the whole
  compressed history (decode kernel for one query token, the tensor-core
  query-chunk path or the masked kernel for more); any other keys go to
  torch's SDPA, as ``_patched_sdpa`` passes non-ChronoQuant caches through.

Usage::

    from chronoquant_mlx_b200 import hf
    hf.register()
    model.set_attn_implementation("chronoquant")
    cache = hf.ChronoQuantHFCache(model.config, **FULL_THROTTLE_V3_CONFIG)
    logits = model(input_ids, past_key_values=cache, use_cache=True).logits
"""

from __future__ import annotations

import torch

from .attention import chronoquant_sdpa
from .cache import ChronoQuantCache

NAME = "chronoquant"
_TAG = "_chronoquant_cache"

try:
    from transformers.cache_utils import Cache, CacheLayerMixin
except ImportError:  # transformers absent: the module imports, the classes raise when built
    Cache = CacheLayerMixin = object


class ChronoQuantLayer(CacheLayerMixin):
    """One transformer layer's compressed KV cache in the transformers cache protocol."""

    is_sliding = False

    def __init__(self, layer_idx: int, **cache_kwargs):
        if CacheLayerMixin is object:
            raise ImportError("transformers is not installed")
        super().__init__()
        self.layer_idx = layer_idx
        self.cache_kwargs = dict(cache_kwargs)
        self.cq = ChronoQuantCache(layer_idx=layer_idx, **self.cache_kwargs)

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.cq.update_and_fetch(key_states, value_states)
        setattr(key_states, _TAG, self.cq)  # read by chronoquant_attention
        return key_states, value_states

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.cq.offset + query_length, 0

    def get_seq_length(self) -> int:
        return self.cq.offset

    def get_max_cache_shape(self) -> int:
        return -1

    def offload(self):
        pass

    def prefetch(self):
        pass

    def reset(self) -> None:
        self.cq = ChronoQuantCache(layer_idx=self.layer_idx, **self.cache_kwargs)
        self.is_initialized = False

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        raise NotImplementedError("ChronoQuant caches are not reorderable (beam search is not supported)")

    def crop(self, max_length: int) -> None:
        raise NotImplementedError("ChronoQuant caches are not trimmable (cache.py:265-266)")


class ChronoQuantHFCache(Cache):
    """A transformers ``Cache`` of ChronoQuant layers.  ``config`` gives the
    layer count (``num_hidden_layers``); keyword arguments are
    ``ChronoQuantCache``'s (strides, bits, dead zones, per_layer_v_bits,
    page_tokens, max_tokens)."""

    def __init__(self, config=None, num_layers: int | None = None, **cache_kwargs):
        if Cache is object:
            raise ImportError("transformers is not installed")
        n = num_layers if num_layers is not None else config.num_hidden_layers
        super().__init__(layers=[ChronoQuantLayer(i, **cache_kwargs) for i in range(n)])

    @property
    def caches(self) -> list:
        """The per-layer ``ChronoQuantCache`` objects (``state``, ``nbytes``, ...)."""
        return [layer.cq for layer in self.layers]

    @property
    def nbytes(self) -> int:
        return sum(c.nbytes for c in self.caches)


def chronoquant_attention(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: torch.Tensor | None, scaling: float | None = None, dropout: float = 0.0,
                          **kwargs):
    """transformers attention function: (attn_output [B, Tq, Hq, D], None)."""
    cache = getattr(key, _TAG, None)
    if cache is None:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query, key, value, attention_mask, scaling=scaling, dropout=dropout,
                                      **kwargs)
    if kwargs.get("sliding_window") is not None:
        raise NotImplementedError("sliding-window attention over a ChronoQuant cache is not supported")
    if dropout:
        raise NotImplementedError("attention dropout is not supported (inference path)")
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    q_len = query.shape[2]
    if attention_mask is None:
        mask = "causal" if q_len > 1 else None
    else:
        mask = attention_mask  # boolean (True = attend) or additive, [B?, H?, Tq, Tk]
    out = chronoquant_sdpa(query, None, None, cache, scaling, mask=mask)
    return out.transpose(1, 2).contiguous(), None


def register(name: str = NAME) -> None:
    """Register ``chronoquant_attention`` (and sdpa-style masks) under ``name``."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(name, chronoquant_attention)
    AttentionMaskInterface.register(name, sdpa_mask)
