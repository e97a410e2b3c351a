"""Optional NVTX ranges around the package's public entry points.

The reference has no tracing (wall-clock prints in off-path scripts only).
Here a profiler timeline (Nsight Systems, or ncu's NVTX filters) can show
which call of the cache protocol issued which kernels: with the environment
variable ``CQ_NVTX=1`` set when the package is imported, ``traced(name)``
wraps a function in ``torch.cuda.nvtx.range_push(name)`` /
``range_pop()``.  Without it the decorator returns the function itself, so
the default path pays nothing.  The ranges are host-side markers: inside a
CUDA-graph capture they mark the capture, not the replays.

Range names: ``cq.append`` (ChronoQuantCache.update_and_fetch), ``cq.sdpa``
(chronoquant_sdpa), ``cq.sdpa_lse`` (chronoquant_sdpa_with_lse),
``cq.reconstruct`` (reconstruct_history), ``cq.graph_step`` /
``cq.graph_replay`` (DecodeGraph), ``cq.seq_exchange`` / ``cq.seq_merge``
(sequence-split partials).
"""

from __future__ import annotations

import functools
import os

ENABLED = os.environ.get("CQ_NVTX", "0") not in ("", "0")


def traced(name: str):
    """Decorator: an NVTX range named ``name`` around each call, when tracing
    is enabled at import time; otherwise the function unchanged."""
    def deco(fn):
        if not ENABLED:
            return fn
        import torch

        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()
        wrapper.__cq_trace__ = name
        return wrapper
    return deco
