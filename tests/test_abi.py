"""The C ABI library loads without a GPU and exports every symbol that
include/chronoquant_b200.h declares; argument validation answers with status
codes and messages (no compute calls here)."""

import ctypes
import os
import re

import pytest

from chronoquant_mlx_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(cq_\w+)\s*\(", src, flags=re.M)
    return names


def test_header_declares_functions():
    names = declared_functions()
    assert "cq_append" in names and "cq_attention" in names and len(names) >= 15


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(name):
    L = _lib.lib()
    assert hasattr(L, name), name


def test_binding_covers_header():
    assert set(declared_functions()) <= set(_lib.EXPORTED) | {"cq_abi_version", "cq_last_error"}


def test_abi_version():
    assert _lib.lib().cq_abi_version() == _lib.CQ_ABI_VERSION == 3
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                            "chronoquant_b200.h")).read()
    assert "#define CQ_ABI_VERSION 3" in hdr


def test_graft_build_entry():
    """The driver's build check: build() compiles (incrementally) and loads the library."""
    import __graft_entry__
    __graft_entry__.build()


def _desc(**over):
    d = _lib.CqPagedCache()
    d.batch, d.kv_heads, d.head_dim, d.page_tokens = 2, 8, 128, 256
    d.max_pages, d.n_pages = 4, 8
    d.block_table = 0x1000  # never dereferenced by validation
    for name, s in (("k", 32), ("v", 8)):
        c = getattr(d, name)
        c.stride, c.bits, c.dead_zone = s, 4, 0.0
        c.anchors_per_page = 256 // s
        c.pframes_per_page = 256 - 256 // s
        c.scale_row = 256
        c.code_order = 0
        c.scale_index = 1
        c.keyframes, c.codes, c.scales = 0x2000, 0x3000, 0x4000
    for k, v in over.items():
        setattr(d, k, v)
    return d


def test_workspace_query_without_gpu():
    d = _desc()
    n = ctypes.c_size_t(0)
    st = _lib.lib().cq_attention_workspace(ctypes.byref(d), 1000, 32, 1, 0, ctypes.byref(n))
    assert st == 0 and n.value > 0


@pytest.mark.parametrize("over,msg", [
    ({"head_dim": 12}, "head_dim"),
    ({"page_tokens": 100}, "multiple of the stride"),
    ({"block_table": None}, "block_table"),
])
def test_validation_errors(over, msg):
    d = _desc(**over)
    n = ctypes.c_size_t(0)
    st = _lib.lib().cq_attention_workspace(ctypes.byref(d), 1000, 32, 1, 0, ctypes.byref(n))
    assert st != 0
    assert msg in _lib.lib().cq_last_error().decode()


def test_append_null_inputs_rejected():
    d = _desc()
    st = _lib.lib().cq_append(ctypes.byref(d), None, 0, 0, 0, None, 0, 0, 0, 0, 0, 1, None)
    assert st == _lib.CQ_ERR_INVALID
    assert "null" in _lib.lib().cq_last_error().decode()


def test_gqa_mismatch_rejected():
    d = _desc()
    n = ctypes.c_size_t(0)
    st = _lib.lib().cq_attention_workspace(ctypes.byref(d), 1000, 12, 1, 0, ctypes.byref(n))
    assert st == _lib.CQ_ERR_INVALID


def test_bits_out_of_range_rejected():
    d = _desc()
    d.v.bits = 1
    n = ctypes.c_size_t(0)
    assert _lib.lib().cq_attention_workspace(ctypes.byref(d), 10, 32, 1, 0, ctypes.byref(n)) == _lib.CQ_ERR_INVALID


def test_check_raises_value_error():
    d = _desc(head_dim=12)
    n = ctypes.c_size_t(0)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.lib().cq_attention_workspace(ctypes.byref(d), 10, 32, 1, 0, ctypes.byref(n)), "x")
