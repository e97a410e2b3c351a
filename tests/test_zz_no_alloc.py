"""cq_attention_static_scratch: attention whose split-KV partials live in the
library's fixed per-device scratch array instead of a caller workspace.

Collected last (file name) so that it also runs after every other GPU test in
the same process; it passes alone in a fresh process too.  Each case makes two
calls in a row through the C ABI and compares both with cq_attention given a
caller-allocated workspace: the same kernels on the same inputs, so the
outputs agree bit for bit (the tests' usual max-abs 2e-3 / relative 1e-2 bar
is checked as well).  The calls must not allocate: device free memory and
the caching allocator's counters stay unchanged across them.  Before the
calls, the shared scratch is filled with the partials of a different shape,
so stale contents (the decode kernel's completion words included) are
exercised.  Finally one call is captured in a CUDA graph and replayed twice."""

import ctypes
import math

import numpy as np
import pytest
import torch

from chronoquant_mlx_b200 import _lib
from oracle import cq_oracle as O

ATOL, RTOL = 2e-3, 1e-2


def _attention(fn_name, desc, T, q, causal, out, lse, ws=None):
    L = _lib.lib()
    qs = q.stride()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    common = (ctypes.byref(desc), T, q.data_ptr(), _lib.CQ_BF16, q.shape[1], q.shape[2], causal, qs[0], qs[1],
              qs[2], 1.0 / math.sqrt(q.shape[3]), out.data_ptr(), _lib.CQ_F32, lse.data_ptr())
    if fn_name == "cq_attention":
        st = L.cq_attention(*common, ws.data_ptr(), ws.numel() * 4, 0, stream)
    else:
        st = L.cq_attention_static_scratch(*common, 0, stream)
    _lib.check(st, fn_name)


def _close(a, b):
    a = a.detach().cpu().double().numpy()
    b = b.detach().cpu().double().numpy()
    err = np.abs(a - b)
    assert (err <= ATOL + RTOL * np.abs(b)).all(), f"max abs err {err.max():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hkv,Hq,T,q_len,stride_k,stride_v", [
    (2, 2, 8, 1000, 1, 32, 8),     # split-KV decode kernel
    (3, 2, 16, 777, 1, 64, 32),    # decode, Full-Throttle strides
    (1, 2, 8, 600, 16, 32, 8),     # causal query chunk (general kernel)
])
def test_static_scratch_matches_workspace_path(B, Hkv, Hq, T, q_len, stride_k, stride_v):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=T + q_len)
    cache = ChronoQuantCache(stride_k=stride_k, stride_v=stride_v)
    cache.update_and_fetch(torch.from_numpy(K).cuda().half(), torch.from_numpy(V).cuda().half())
    desc = cache.store.descriptor()
    gen = torch.Generator(device="cpu").manual_seed(T)
    qs = [(torch.randn((B, Hq, q_len, 128), generator=gen) / math.sqrt(128)).to(torch.bfloat16).cuda()
          for _ in range(2)]
    causal = 1 if q_len > 1 else 0

    need = ctypes.c_size_t(0)
    _lib.check(_lib.lib().cq_attention_workspace(ctypes.byref(desc), T, Hq, q_len, 0, ctypes.byref(need)), "ws")
    assert 0 < need.value <= _lib.CQ_STATIC_SCRATCH_BYTES
    ws = torch.empty((need.value + 3) // 4, dtype=torch.float32, device="cuda")
    ref = []
    for q in qs:
        o = torch.empty((B, Hq, q_len, 128), dtype=torch.float32, device="cuda")
        lse = torch.empty((B, Hq, q_len), dtype=torch.float32, device="cuda")
        _attention("cq_attention", desc, T, q, causal, o, lse, ws)
        ref.append((o, lse))

    outs = [(torch.empty((B, Hq, q_len, 128), dtype=torch.float32, device="cuda"),
             torch.empty((B, Hq, q_len), dtype=torch.float32, device="cuda")) for _ in qs]
    # leave other partials in the shared scratch first: a decode of another shape
    other = ChronoQuantCache(stride_k=32, stride_v=8)
    Ko, Vo = O.ar1_kv(1, 8, 3000, 128, seed=5)
    other.update_and_fetch(torch.from_numpy(Ko).cuda().half(), torch.from_numpy(Vo).cuda().half())
    qo = torch.randn((1, 32, 1, 128), generator=gen).to(torch.bfloat16).cuda()
    oo = torch.empty((1, 32, 1, 128), dtype=torch.float32, device="cuda")
    lo = torch.empty((1, 32, 1), dtype=torch.float32, device="cuda")
    _attention("cq_attention_static_scratch", other.store.descriptor(), 3000, qo, 0, oo, lo)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    stats0 = torch.cuda.memory_stats()
    for q, (o, lse) in zip(qs, outs):  # two calls in a row on the same scratch
        _attention("cq_attention_static_scratch", desc, T, q, causal, o, lse)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    stats1 = torch.cuda.memory_stats()
    for k in ("allocation.all.allocated", "segment.all.allocated"):
        assert stats1.get(k, 0) == stats0.get(k, 0), k
    for (o, lse), (ro, rlse) in zip(outs, ref):
        assert torch.isfinite(o).all()
        _close(o, ro)
        _close(lse, rlse)
        assert torch.equal(o, ro) and torch.equal(lse, rlse)

    # after the first call the entry point is capture-safe: one call captured in a CUDA graph
    # (the completion-word clear and the kernels), replayed twice, gives the same bits
    go = torch.zeros_like(outs[0][0])
    gl = torch.zeros_like(outs[0][1])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _attention("cq_attention_static_scratch", desc, T, qs[0], causal, go, gl)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        go.zero_()
        gl.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(go, ref[0][0]) and torch.equal(gl, ref[0][1])
    assert torch.cuda.mem_get_info()[0] == free1
    del graph


def test_static_scratch_rejects_oversized_shape():
    """A shape whose partials exceed the fixed scratch is refused before any
    device work (no GPU needed): a 2048-token causal chunk over 32 heads needs
    65536 rows of partials."""
    d = _lib.CqPagedCache()
    d.batch, d.kv_heads, d.head_dim, d.page_tokens = 1, 8, 128, 256
    d.max_pages, d.n_pages = 16, 16
    d.block_table = 0x1000  # never dereferenced on this path
    for name, s in (("k", 32), ("v", 8)):
        c = getattr(d, name)
        c.stride, c.bits, c.dead_zone = s, 4, 0.0
        c.anchors_per_page, c.pframes_per_page = 256 // s, 256 - 256 // s
        c.scale_row, c.code_order, c.scale_index = 256, _lib.CQ_ORDER_NATURAL, _lib.CQ_SCALE_BY_TOKEN
        c.keyframes, c.codes, c.scales = 0x2000, 0x3000, 0x4000
    L = _lib.lib()
    st = L.cq_attention_static_scratch(ctypes.byref(d), 4096, 0x5000, _lib.CQ_BF16, 32, 2048, 1, 0, 0, 0, 1.0,
                                       0x6000, _lib.CQ_F32, None, 0, None)
    assert st == _lib.CQ_ERR_WORKSPACE
    msg = L.cq_last_error().decode()
    assert "more than the fixed" in msg and str(_lib.CQ_STATIC_SCRATCH_BYTES) in msg
