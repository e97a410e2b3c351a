"""Small torch <-> C-ABI helpers shared by the package modules."""

from __future__ import annotations

import torch

from . import _lib

_DT = {torch.float16: _lib.CQ_F16, torch.bfloat16: _lib.CQ_BF16, torch.float32: _lib.CQ_F32}


def cq_dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float16, bfloat16 or float32") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    """The B200 path has no CPU fallback: every tensor must live on a CUDA device."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("chronoquant_mlx_b200 computes on CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
