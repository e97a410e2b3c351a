"""ctypes binding of libchronoquant_b200.so (the C ABI in include/chronoquant_b200.h).

The shared library is built in-tree by ``chronoquant_mlx_b200.build`` (or
``__graft_entry__.build()``).  There is no fallback: if the library is
missing, importing the package's compute entry points raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# CQ_CHECKS=1 at import selects the bounds-checked debug build (build.py --checks)
CHECKS = os.environ.get("CQ_CHECKS", "0") not in ("", "0")
LIB_PATH = os.path.join(_HERE, "libchronoquant_b200_checks.so" if CHECKS else "libchronoquant_b200.so")

CQ_OK = 0
CQ_ERR_INVALID = -1
CQ_ERR_UNSUPPORTED = -2
CQ_ERR_CUDA = -3
CQ_ERR_WORKSPACE = -4

CQ_ABI_VERSION = 3  # CQ_ABI_VERSION of include/chronoquant_b200.h
CQ_F16, CQ_BF16, CQ_F32 = 0, 1, 2
CQ_ORDER_NATURAL, CQ_ORDER_MMA, CQ_ORDER_PLANES3, CQ_ORDER_PLANES2 = 0, 1, 2, 3
CQ_SCALE_BY_PFRAME, CQ_SCALE_BY_TOKEN = 0, 1
CQ_STATIC_SCRATCH_BYTES = 8 << 20  # cq_attention_static_scratch's fixed per-device scratch

EXPORTED = [
    "cq_abi_version", "cq_last_error", "cq_device_error", "cq_append", "cq_attention", "cq_attention_workspace",
    "cq_attention_masked", "cq_lse_merge", "cq_lse_merge_packed", "cq_reconstruct", "cq_export_state", "cq_import_state", "cq_quantize_delta",
    "cq_dequantize_delta", "cq_pack_int4", "cq_unpack_int4", "cq_sdpa_reference_layout",
    "cq_sdpa_reference_layout_workspace", "cq_attention_static_scratch", "cq_decode_chunk_tokens",
    "cq_append_at", "cq_attention_at", "cq_decode_step_at", "cq_prefill_prepare", "cq_prefill_attend",
    "cq_rmsnorm", "cq_qk_norm_rope", "cq_silu_mul", "cq_peer_sum_norm", "cq_peer_region_bytes",
    "cq_peer_region_alloc", "cq_peer_region_open", "cq_peer_region_close", "cq_peer_region_free",
]


class CqComponent(ctypes.Structure):
    _fields_ = [
        ("stride", ctypes.c_int32), ("bits", ctypes.c_int32), ("dead_zone", ctypes.c_float),
        ("anchors_per_page", ctypes.c_int32), ("pframes_per_page", ctypes.c_int32),
        ("scale_row", ctypes.c_int32), ("code_order", ctypes.c_int32), ("scale_index", ctypes.c_int32),
        ("keyframes", ctypes.c_void_p), ("codes", ctypes.c_void_p), ("scales", ctypes.c_void_p),
        ("keyframe_head_stride", ctypes.c_int64), ("code_head_stride", ctypes.c_int64),
        ("scale_head_stride", ctypes.c_int64), ("chunk_tokens", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("keyframe_chunk_stride", ctypes.c_int64), ("code_chunk_stride", ctypes.c_int64),
        ("scale_chunk_stride", ctypes.c_int64),
    ]


class CqPagedCache(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("page_tokens", ctypes.c_int32), ("max_pages", ctypes.c_int32), ("n_pages", ctypes.c_int32),
        ("block_table", ctypes.c_void_p), ("k", CqComponent), ("v", CqComponent),
    ]


class CudaLibError(RuntimeError):
    pass


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P, I32, I64, F, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    C = ctypes.POINTER(CqPagedCache)
    lib.cq_abi_version.restype = ctypes.c_int
    lib.cq_abi_version.argtypes = []
    lib.cq_last_error.restype = ctypes.c_char_p
    lib.cq_last_error.argtypes = []
    sig = {
        "cq_device_error": [ctypes.POINTER(ctypes.c_int), ctypes.c_int],
        "cq_append": [C, P, I64, I64, I64, P, I64, I64, I64, ctypes.c_int, I64, I32, P],
        "cq_attention": [C, I64, P, ctypes.c_int, I32, I32, I32, I64, I64, I64, F, P, ctypes.c_int, P, P, SZ, I32,
                         P],
        "cq_attention_workspace": [C, I64, I32, I32, I32, ctypes.POINTER(SZ)],
        "cq_attention_masked": [C, I64, P, ctypes.c_int, I32, I32, I64, I64, I64, F, P, ctypes.c_int, ctypes.c_int,
                                I64, I64, I64, I64, P, ctypes.c_int, P, SZ, I32, P],
        "cq_lse_merge": [P, P, I32, I64, I32, P, ctypes.c_int, P],
        "cq_lse_merge_packed": [P, I32, I64, I32, P, ctypes.c_int, P],
        "cq_reconstruct": [C, ctypes.c_int, I64, P, ctypes.c_int, P],
        "cq_export_state": [C, ctypes.c_int, I64, P, P, P, P],
        "cq_import_state": [C, ctypes.c_int, I64, P, P, P, P],
        "cq_quantize_delta": [P, ctypes.c_int, I64, I32, I32, F, P, P, P],
        "cq_dequantize_delta": [P, P, I64, I32, P, P],
        "cq_pack_int4": [P, I64, I32, P, P],
        "cq_unpack_int4": [P, I64, I32, P, P],
        "cq_sdpa_reference_layout": [P, I32, I32, P, I32, P, P, I32, P, I32, P, P, I32, I32, I64, I32, I32, P, P,
                                     SZ, P],
        "cq_sdpa_reference_layout_workspace": [I32, I32, I64, ctypes.POINTER(SZ)],
        "cq_decode_chunk_tokens": [I32, I32, I32, I32],
        "cq_append_at": [C, P, I64, I64, I64, P, I64, I64, I64, ctypes.c_int, P, I32, P],
        "cq_attention_at": [C, P, I64, P, ctypes.c_int, I32, I64, I64, F, P, ctypes.c_int, P, P, SZ, P],
        "cq_decode_step_at": [C, P, I64, I64, P, I64, I64, ctypes.c_int, P, I64, P, ctypes.c_int, I32, I64, I64, F, P,
                              ctypes.c_int, P, P, SZ, P],
        "cq_rmsnorm": [P, P, P, I64, I32, F, ctypes.c_int, P],
        "cq_qk_norm_rope": [P, I64, I32, I32, I32, I32, P, P, P, P, F, P, P, P, ctypes.c_int, P],
        "cq_silu_mul": [P, P, I64, I32, ctypes.c_int, P],
        "cq_prefill_prepare": [C, I64, P, ctypes.c_int, I32, I32, I64, I64, I64, F, P, SZ, P],
        "cq_prefill_attend": [C, I64, I32, I32, I32, P, ctypes.c_int, P, P, SZ, P],
        "cq_attention_static_scratch": [C, I64, P, ctypes.c_int, I32, I32, I32, I64, I64, I64, F, P, ctypes.c_int,
                                        P, I32, P],
        "cq_peer_sum_norm": [ctypes.POINTER(ctypes.c_uint64), I32, I32, I32, I64, I64, I32, P, P, P, F, P, P,
                             ctypes.c_int, P],
        "cq_peer_region_alloc": [I64, ctypes.POINTER(P), P],
        "cq_peer_region_open": [P, ctypes.POINTER(P)],
        "cq_peer_region_close": [P],
        "cq_peer_region_free": [P],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    lib.cq_peer_region_bytes.restype = I64
    lib.cq_peer_region_bytes.argtypes = [I64, I32, I32]
    return lib


def lib():
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{os.path.basename(LIB_PATH)} not found at {LIB_PATH}; build it with "
                    f"`python -m chronoquant_mlx_b200.build{' --checks' if CHECKS else ''}` (nvcc, sm_100a). "
                    "There is no CPU fallback.")
            _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def check(status: int, what: str = "") -> None:
    """Raise on a non-zero status from the C ABI."""
    if status == CQ_OK:
        return
    msg = (lib().cq_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status in (CQ_ERR_INVALID, CQ_ERR_WORKSPACE):
        raise ValueError(text)
    if status == CQ_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise CudaLibError(text)
