"""Physical 3-bit and 2-bit V codes (``ChronoQuantCache(v_pack=3)`` and
``v_pack=2``): opt-in store formats that keep V codes of 3 (2) bits or fewer
in 3 (2) bits per value (two bit planes, 48 bytes per row at head_dim 128, or
one plane of 32 bytes) instead of the INT4 lanes the reference uses
(README.md:57).  The codes themselves are the reference's
(codec.py:23-65), so everything observable through the reference API is
unchanged: the state export (INT4 lanes), the fp16 reconstruction and the
attention.  Checked against the oracle; the physical rows against the
oracle's own bit-plane packing."""

import math

import numpy as np
import pytest
import torch

from oracle import cq_oracle as O

ATOL, RTOL = 2e-3, 1e-2


def test_oracle_planes_roundtrip_and_int4_equivalence():
    rng = np.random.default_rng(3)
    codes = rng.integers(-4, 4, size=(2, 3, 5, 128)).astype(np.int8)
    rows = O.pack_planes3(codes)
    assert rows.shape == (2, 3, 5, 12) and rows.dtype == np.uint32
    assert np.array_equal(O.unpack_planes3(rows, 128), codes)
    # the bit positions: with g = d % 8, k = d // 8, the low bits of dim d at word g, bit 2k; its high
    # bit at word 8 + g // 2, bit 16 (g % 2) + k
    for d in (0, 37, 127):
        c = np.full((1, 128), -4, np.int8)
        c[0, d] = 3  # v = 7
        r = O.pack_planes3(c)
        g, k = d % 8, d // 8
        expect = np.zeros(12, np.uint32)
        expect[g] = 3 << (2 * k)
        expect[8 + g // 2] = 1 << (16 * (g % 2) + k)
        assert np.array_equal(r[0], expect), d


def test_oracle_planes2_roundtrip():
    rng = np.random.default_rng(4)
    codes = rng.integers(-2, 2, size=(2, 3, 5, 128)).astype(np.int8)
    rows = O.pack_planes2(codes)
    assert rows.shape == (2, 3, 5, 8) and rows.dtype == np.uint32
    assert np.array_equal(O.unpack_planes2(rows, 128), codes)
    for d in (0, 37, 127):
        c = np.full((1, 128), -2, np.int8)
        c[0, d] = 1  # v = 3
        expect = np.zeros(8, np.uint32)
        expect[d % 8] = 3 << (2 * (d // 8))
        assert np.array_equal(O.pack_planes2(c)[0], expect), d


def test_cache_options():
    from chronoquant_mlx_b200 import ChronoQuantCache
    with pytest.raises(ValueError):
        ChronoQuantCache(v_pack=5)
    with pytest.raises(ValueError):
        ChronoQuantCache(delta_bits_v=4, v_pack=3)  # 4-bit codes do not fit 3 bits
    with pytest.raises(ValueError):
        ChronoQuantCache(delta_bits_v=3, v_pack=2)
    assert ChronoQuantCache(delta_bits_v=2, v_pack=2).v_pack == 2
    c = ChronoQuantCache(stride_k=64, stride_v=32, delta_bits_v=3, v_pack=3)
    assert "v_pack=3" in c.meta_state
    d = ChronoQuantCache()
    d.meta_state = c.meta_state
    assert d.v_pack == 3 and d.delta_bits_v == 3


def _cache_pair(B, H, T, chunks, v_pack=3, **kw):
    from chronoquant_mlx_b200 import ChronoQuantCache
    K, V = O.ar1_kv(B, H, T, 128, rho_k=0.97, rho_v=0.85, seed=T)
    g = ChronoQuantCache(v_pack=v_pack, **kw)
    o = O.OracleCache(**kw)
    t = 0
    for n in chunks:
        g.update_and_fetch(torch.from_numpy(K[:, :, t:t + n]).cuda(), torch.from_numpy(V[:, :, t:t + n]).cuda())
        o.update_and_fetch(K[:, :, t:t + n], V[:, :, t:t + n])
        t += n
    return g, o, K, V


def _physical_v_rows(cache, b, h):
    """V code rows of (sequence b, kv-head h) read straight from the page pool,
    in P-frame order: uint32 [n_pframes, row words]."""
    st = cache.store
    comp = st.comps[1]
    table = st.block_table.cpu().numpy()
    buf = st.buf[:, h].cpu().numpy()
    rows = []
    for t in range(cache.offset):
        if t % comp.stride == 0:
            continue
        lp, tl = divmod(t, st.P)
        j, x = divmod(tl, st.chunk)
        a = x // comp.stride
        r = x - a - 1
        off = j * st.chunk_bytes + comp.off_cd + r * comp.row_words * 4
        rows.append(buf[table[b, lp], off:off + comp.row_words * 4].view(np.uint32))
    return np.stack(rows)


@pytest.mark.gpu
@pytest.mark.parametrize("v_pack,kw,chunks", [
    (3, dict(stride_k=64, stride_v=32, delta_bits_k=4, delta_bits_v=3, dead_zone_v=0.05), [600, 1, 1, 97, 1]),
    (3, dict(stride_k=32, stride_v=8, delta_bits_v=3, dead_zone_v=0.0), [300, 5, 1]),
    (3, dict(stride_k=32, stride_v=8, per_layer_v_bits=[2], dead_zone_v=0.2), [257, 33]),
    (2, dict(stride_k=64, stride_v=32, delta_bits_k=4, delta_bits_v=2, dead_zone_v=0.05), [600, 1, 1, 97, 1]),
    (2, dict(stride_k=32, stride_v=8, delta_bits_v=2, dead_zone_v=0.0), [300, 5, 1]),
    (2, dict(stride_k=16, stride_v=16, delta_bits_v=2, dead_zone_v=0.2), [257, 33]),
])
def test_pack_matches_oracle(v_pack, kw, chunks):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import chronoquant_sdpa
    B, H, Hq = 2, 2, 8
    T = sum(chunks)
    g, o, K, V = _cache_pair(B, H, T, chunks, v_pack=v_pack, **kw)
    # the reference-layout state (INT4 lanes) and the fp16 reconstruction, bit for bit
    for a, r in zip(g.state, o.state):
        a = a.cpu()
        a = a.view(torch.int32).numpy().view(np.uint32) if a.dtype == torch.uint32 else a.numpy()
        assert np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(r).view(np.uint8))
    fk, fv = o.reconstruct_history()
    gk, gv = (t.cpu().numpy() for t in g.reconstruct_history())
    assert np.array_equal(gk.view(np.uint16), fk.view(np.uint16))
    assert np.array_equal(gv.view(np.uint16), fv.view(np.uint16))
    # the physical rows are the oracle's codes in bit planes
    _, pv, _ = o.active("v")
    pack = O.pack_planes3 if v_pack == 3 else O.pack_planes2
    for b, h in ((0, 0), (1, 1)):
        codes = O.unpack_int4(pv[b, h], 128)
        assert np.array_equal(_physical_v_rows(g, b, h), pack(codes))
    # bytes: the reference accounting is unchanged; the store holds 16 (32) bytes less per V P-frame row
    npf_v = T - O.num_keyframes(T, kw["stride_v"])
    assert g.physical_nbytes == g.nbytes - B * H * npf_v * (64 - 16 * v_pack)
    # attention (decode: the sm_100a decode kernel for strides (64, 32) and (32, 8), else the general
    # kernel; the causal chunk: the general kernel) against exact float64
    scale = 1.0 / math.sqrt(128)
    k32, v32 = o.reconstruct_history_f32()
    for q_len, causal in ((1, False), (16, True)):
        q = (np.random.default_rng(q_len).standard_normal((B, Hq, q_len, 128)) / math.sqrt(128)).astype(np.float16)
        out = chronoquant_sdpa(torch.from_numpy(q).cuda(), None, None, g, scale, mask="causal" if causal else None)
        qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
        ref = O.exact_sdpa(qs, k32, v32, causal)
        err = np.abs(out.float().cpu().numpy() - ref)
        assert (err <= ATOL + RTOL * np.abs(ref)).all(), float(err.max())


@pytest.mark.gpu
@pytest.mark.parametrize("v_pack", [3, 2])
def test_pack_state_roundtrip(v_pack):
    """state exported from a v_pack=3 (2) cache (INT4 lanes, the reference
    layout) and imported into another such cache gives the same physical
    pool."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache
    kw = dict(stride_k=64, stride_v=32, delta_bits_v=v_pack)
    g, _, _, _ = _cache_pair(1, 2, 500, [500], v_pack=v_pack, **kw)
    c2 = ChronoQuantCache(v_pack=v_pack, **kw)
    c2.state = g.state
    assert c2.offset == g.offset
    for b, h in ((0, 0), (0, 1)):
        assert np.array_equal(_physical_v_rows(c2, b, h), _physical_v_rows(g, b, h))
    for a, b in zip(g.state, c2.state):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
