"""ChronoQuant KV-cache codec and fused dequant-attention, B200-native.

Drop-in for the reference package ``chronoquant_mlx`` on PyTorch CUDA
tensors: the same public names (``__init__.py:1-21`` of the reference) backed
by hand-written sm_100a CUDA kernels behind a C ABI
(``include/chronoquant_b200.h``, ``libchronoquant_b200.so``).
"""

from .cache import ChronoQuantCache
from .patch import (
    FULL_THROTTLE_V3_CONFIG,
    apply,
    apply_patch,
    create_chronoquant_caches,
    create_full_throttle_caches,
    revert,
)
from .attention import chronoquant_sdpa
from .graph import DecodeGraph
from .prompt_cache import load_prompt_cache, save_prompt_cache

__all__ = [
    "ChronoQuantCache",
    "FULL_THROTTLE_V3_CONFIG",
    "apply",
    "apply_patch",
    "create_chronoquant_caches",
    "create_full_throttle_caches",
    "chronoquant_sdpa",
    "DecodeGraph",
    "save_prompt_cache",
    "load_prompt_cache",
]
