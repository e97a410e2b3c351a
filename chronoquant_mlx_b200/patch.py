"""Attention patch and cache factories (patch.py:1-104 of the reference).

``apply()`` replaces the host model's module-level SDPA symbol with a
dispatcher that sends ChronoQuant caches to ``chronoquant_sdpa`` and every
other cache to the original (patch.py:12-33).  The patched symbol is
``chronoquant_mlx_b200.base.scaled_dot_product_attention`` and, like the
reference, its rebinding in every already-imported module under the model
package prefixes (``chronoquant_mlx_b200.models.`` and, when importable,
``mlx_lm.models.``).  Modules imported later keep the original symbol.
"""

from __future__ import annotations

import logging
import sys

from . import base as _base
from .attention import chronoquant_sdpa
from .cache import ChronoQuantCache

log = logging.getLogger("chronoquant_mlx_b200.patch")

_original_sdpa = _base.scaled_dot_product_attention
_patched = False
MODEL_PREFIXES = ["chronoquant_mlx_b200.models."]


def _patched_sdpa(queries, keys, values, cache, scale, mask, **kwargs):
    if isinstance(cache, ChronoQuantCache):
        return chronoquant_sdpa(queries, keys, values, cache, scale, mask)
    return _original_sdpa(queries, keys, values, cache, scale, mask, **kwargs)


def _targets():
    mods = [_base]
    mlx_base = sys.modules.get("mlx_lm.models.base")
    if mlx_base is not None:
        mods.append(mlx_base)
    prefixes = list(MODEL_PREFIXES) + (["mlx_lm.models."] if mlx_base is not None else [])
    for name, module in list(sys.modules.items()):
        if module is None or module in mods:
            continue
        if any(name.startswith(p) for p in prefixes) and hasattr(module, "scaled_dot_product_attention"):
            mods.append(module)
    return mods


def apply_patch():
    """Activate the ChronoQuant SDPA dispatch.  Idempotent (patch.py:18-33)."""
    global _patched
    if _patched:
        return
    for module in _targets():
        module.scaled_dot_product_attention = _patched_sdpa
    _patched = True
    # transformers models select attention by name: register "chronoquant" when it is installed
    try:
        from . import hf
        hf.register()
    except ImportError:
        pass
    log.info("ChronoQuant SDPA patch applied to all loaded model modules.")


def apply():
    apply_patch()


def revert():
    """Restore the base symbol (patch.py:40-43 restores only the base module)."""
    global _patched
    _base.scaled_dot_product_attention = _original_sdpa
    _patched = False


def create_chronoquant_caches(model, stride_k: int = 32, stride_v: int = 8, delta_bits_k: int = 4,
                              delta_bits_v: int = 4, dead_zone_k: float = 0.0, dead_zone_v: float = 0.05,
                              use_fused: bool = True, per_layer_v_bits: list = None, **cache_kwargs):
    """Replace every plain ``KVCache`` slot of ``model.make_cache()`` (or
    ``make_prompt_cache(model)``) with a ``ChronoQuantCache`` (patch.py:46-78).

    ``per_layer_v_bits``: V bit width per layer index; slot i gets
    ``delta_bits_v=per_layer_v_bits[i]`` when i is in range, and every cache
    keeps the list (its V codec resolves bits from it, cache.py:192-196).
    Extra keyword arguments (``page_tokens``, ``max_tokens``) go to each cache."""
    caches = model.make_cache() if hasattr(model, "make_cache") else _base.make_prompt_cache(model)
    kv_types = (_base.KVCache,)
    mlx_cache = sys.modules.get("mlx_lm.models.cache")
    if mlx_cache is not None and hasattr(mlx_cache, "KVCache"):
        kv_types = kv_types + (mlx_cache.KVCache,)
    for index in range(len(caches)):
        if isinstance(caches[index], kv_types):
            v_bits = (per_layer_v_bits[index] if per_layer_v_bits and index < len(per_layer_v_bits)
                      else delta_bits_v)
            caches[index] = ChronoQuantCache(stride_k=stride_k, stride_v=stride_v, delta_bits_k=delta_bits_k,
                                             delta_bits_v=v_bits, dead_zone_k=dead_zone_k, dead_zone_v=dead_zone_v,
                                             use_fused=use_fused, per_layer_v_bits=per_layer_v_bits, **cache_kwargs)
            caches[index].layer_idx = index
    return caches


FULL_THROTTLE_V3_CONFIG = {
    "stride_k": 64,
    "stride_v": 32,
    "delta_bits_k": 4,
    "delta_bits_v": 3,
    "dead_zone_k": 0.0,
    "dead_zone_v": 0.05,
}


def create_full_throttle_caches(model, use_fused: bool = True, **cache_kwargs):
    """The Full-Throttle V3 preset (patch.py:81-104): K stride 64 INT4, V
    stride 32 3-bit codes in INT4 lanes, V dead zone 0.05."""
    return create_chronoquant_caches(model, use_fused=use_fused, **FULL_THROTTLE_V3_CONFIG, **cache_kwargs)
