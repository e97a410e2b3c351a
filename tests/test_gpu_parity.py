"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the
fixtures generated from the reference.

Bars: packed codes, scales, anchors and the fp16 reconstruction bit-exact;
attention within max-abs 2e-3 / relative 1e-2 (numpy.allclose atol=2e-3,
rtol=1e-2) of the path the reference dispatches to, and within 3e-4 / 3e-3 of
exact float64 attention on the same decoded values for fp32 outputs."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import cq_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import chronoquant_mlx_b200._lib as L
    L.lib()  # fails loudly when the library is missing


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def npy(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


def bits16(a):
    return np.ascontiguousarray(a).view(np.uint16)


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def check_state(cache, g, prefix=""):
    names = ["kf_k", "kf_v", "packed_k", "scales_k", "packed_v", "scales_v"]
    st = cache.state
    assert len(st) == sum(1 for n in names if prefix + n in g.files)
    for n, t in zip(names, st):
        a = npy(t)
        ref = g[prefix + n]
        assert a.shape == ref.shape, n
        assert np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(ref).view(np.uint8)), n


def close(out, ref, atol=ATOL, rtol=RTOL):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(out - ref)
    ok = err <= atol + rtol * np.abs(ref)
    assert ok.all(), f"max abs err {err.max():.3e}, worst rel {(err / (np.abs(ref) + 1e-12)).max():.3e}"


# ---------------------------------------------------------------------------- codec


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("dz", [0.0, 0.05, 0.2, 0.5])
def test_codec_matches_reference_fixture(golden_dir, bits, dz):
    from chronoquant_mlx_b200.codec import ChronoQuantCodec
    g = load(golden_dir, "codec_kat.npz")
    tag = f"b{bits}_dz{int(round(dz * 100)):03d}"
    c = ChronoQuantCodec(stride=8, delta_bits=bits, dead_zone_ratio=dz)
    codes, scale = c.quantize_delta(cu(g["delta"]))
    assert np.array_equal(npy(codes), g[f"codes_{tag}"])
    assert np.array_equal(bits16(npy(scale)), bits16(g[f"scale_{tag}"]))
    deq = c.dequantize_delta(codes, scale)
    assert np.array_equal(bits16(npy(deq)), bits16(g[f"deq_{tag}"]))


def test_codec_bf16_matches_oracle():
    from chronoquant_mlx_b200.codec import ChronoQuantCodec
    gen = np.random.default_rng(3)
    d = (gen.standard_normal((3, 40, 128)) * gen.choice([1e-3, 0.3, 20.0], size=(3, 40, 1))).astype(np.float32)
    d = O.round_bf16(d)
    for bits, dz in ((4, 0.0), (3, 0.05), (2, 0.3)):
        codes, scale = ChronoQuantCodec(delta_bits=bits, dead_zone_ratio=dz).quantize_delta(cu(d, torch.bfloat16))
        rc, rs = O.quantize_delta(d, bits, dz, dtype="bf16")
        assert np.array_equal(npy(codes), rc)
        assert np.array_equal(bits16(npy(scale)), bits16(rs))


def test_zero_residual_rows_give_zero_codes():
    from chronoquant_mlx_b200.codec import ChronoQuantCodec
    d = torch.zeros((2, 128), dtype=torch.float16, device="cuda")
    codes, scale = ChronoQuantCodec().quantize_delta(d)
    assert int(codes.abs().max()) == 0 and float(scale.abs().max()) == 0.0


def test_pack_unpack_reference_fixture(golden_dir):
    from chronoquant_mlx_b200.kernels import pack_int4_codes, unpack_int4_codes
    g = load(golden_dir, "pack_kat.npz")
    assert np.array_equal(npy(pack_int4_codes(cu(g["codes"]))), g["packed"])
    assert np.array_equal(npy(unpack_int4_codes(cu(g["packed"].view(np.int32)).view(torch.uint32), 128)),
                          g["unpacked"])
    assert np.array_equal(npy(pack_int4_codes(cu(g["codes72"]))), g["packed72"])
    assert np.array_equal(npy(unpack_int4_codes(cu(g["packed72"].view(np.int32)).view(torch.uint32), 72)),
                          g["unpacked72"])
    assert np.array_equal(npy(unpack_int4_codes(cu(g["words"].view(np.int32)).view(torch.uint32), 128)),
                          g["words_unpacked"])


# ---------------------------------------------------------------------------- cache


def build_cache(K, V, chunks, dtype=torch.float16, **kw):
    from chronoquant_mlx_b200 import ChronoQuantCache
    c = ChronoQuantCache(**kw)
    t = 0
    for n in chunks:
        kk, vv = c.update_and_fetch(cu(K[:, :, t:t + n], dtype), cu(V[:, :, t:t + n], dtype))
        assert kk.shape[2] == n
        t += n
    return c


def test_reference_test_scenario(golden_dir):
    g = load(golden_dir, "cache_reftest.npz")
    c = build_cache(g["keys"], g["values"], [9], stride_k=4, stride_v=2, delta_bits_k=4, delta_bits_v=4)
    check_state(c, g)
    assert c.nbytes == int(g["nbytes"])
    rk, rv = c.reconstruct_history()
    assert np.array_equal(bits16(npy(rk)), bits16(g["recon_k"]))
    assert np.array_equal(bits16(npy(rv)), bits16(g["recon_v"]))
    # the reference test's own bar against its manual codec
    assert np.abs(npy(rk).astype(np.float32) - g["manual_k"].astype(np.float32)).max() < 1e-3


def test_fused_generation_scenario(golden_dir):
    from chronoquant_mlx_b200 import chronoquant_sdpa
    from chronoquant_mlx_b200.kernels import chronoquant_sdpa_kernel
    g = load(golden_dir, "cache_reftest.npz")
    c = build_cache(g["keys11"], g["values11"], [11], stride_k=4, stride_v=2, delta_bits_k=4, delta_bits_v=4)
    check_state(c, g, "c11_")
    scale = 1.0 / math.sqrt(128)
    q = cu(g["q11"])
    out = chronoquant_sdpa(q, None, None, c, scale, mask=None)
    close(npy(out).astype(np.float32), g["fused11"].astype(np.float32))
    # reference test bar: fused vs reference SDPA over the reconstruction < 2e-2
    assert np.abs(npy(out).astype(np.float32) - g["refsdpa11"].astype(np.float32)).max() < 2e-2
    # the reference-layout kernel entry with the cache's B=1 views
    qs = (q * scale).reshape(4, 128).float()
    ref_layout = chronoquant_sdpa_kernel(qs, c.kernel_keyframes_k(), c.kernel_packed_k(), c.kernel_scales_k(),
                                         c.kernel_keyframes_v(), c.kernel_packed_v(), c.kernel_scales_v(),
                                         c.offset, 4, 2)
    kk, pk, sk = [npy(x) for x in c._export("k")]
    kv, pv, sv = [npy(x) for x in c._export("v")]
    exact = O.fused_decode(npy(qs), kk[0], pk[0], sk[0], kv[0], pv[0], sv[0], c.offset, 4, 2, 128)
    close(npy(ref_layout), exact, atol=1e-5, rtol=1e-4)
    close(npy(out).astype(np.float32).reshape(4, 128), exact)


def test_standard_multi_call(golden_dir):
    from chronoquant_mlx_b200 import chronoquant_sdpa
    g = load(golden_dir, "cache_standard.npz")
    from chronoquant_mlx_b200 import ChronoQuantCache
    c = ChronoQuantCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
    t = 0
    for n, nb in zip(g["chunks"], g["nbytes_after"]):
        c.update_and_fetch(cu(g["K"][:, :, t:t + n]), cu(g["V"][:, :, t:t + n]))
        t += int(n)
        assert c.nbytes == int(nb)
    check_state(c, g)
    rk, rv = c.reconstruct_history()
    assert np.array_equal(bits16(npy(rk)), bits16(g["recon_k"]))
    assert np.array_equal(bits16(npy(rv)), bits16(g["recon_v"]))
    scale = 1.0 / math.sqrt(128)
    out = chronoquant_sdpa(cu(g["q1"]), None, None, c, scale, mask=None)  # B=2: the reference's fallback
    close(npy(out), g["sdpa_q1_fallback"])
    c.update_and_fetch(cu(g["K"][:, :, t:t + 4]), cu(g["V"][:, :, t:t + 4]))
    check_state(c, g, "final_")
    mask = c.make_mask(4)
    assert mask == "causal"
    out4 = chronoquant_sdpa(cu(g["q4"]), None, None, c, scale, mask=mask)
    close(npy(out4), g["sdpa_q4_causal"])
    # explicit boolean mask array == implicit causal rule
    arr = c.make_mask(4, return_array=True)
    out4b = chronoquant_sdpa(cu(g["q4"]), None, None, c, scale, mask=arr)
    assert np.array_equal(bits16(npy(out4b)), bits16(npy(out4)))
    # additive mask of zeros == no mask
    zero = torch.zeros((4, c.offset), dtype=torch.float32, device="cuda")
    a = chronoquant_sdpa(cu(g["q4"]), None, None, c, scale, mask=zero)
    b = chronoquant_sdpa(cu(g["q4"]), None, None, c, scale, mask=None)
    assert np.array_equal(bits16(npy(a)), bits16(npy(b)))


def test_ftv3(golden_dir):
    from chronoquant_mlx_b200 import FULL_THROTTLE_V3_CONFIG, chronoquant_sdpa
    from chronoquant_mlx_b200.attention import chronoquant_sdpa_with_lse
    g = load(golden_dir, "cache_ftv3.npz")
    c = build_cache(g["K"], g["V"], [int(x) for x in g["chunks"]], **FULL_THROTTLE_V3_CONFIG)
    check_state(c, g)
    assert c.nbytes == int(g["nbytes"])
    rk, rv = c.reconstruct_history()
    assert np.array_equal(bits16(npy(rk)), bits16(g["recon_k"]))
    assert np.array_equal(bits16(npy(rv)), bits16(g["recon_v"]))
    scale = 1.0 / math.sqrt(128)
    out = chronoquant_sdpa(cu(g["q1"]), None, None, c, scale)
    close(npy(out).astype(np.float32), g["sdpa_fused"].astype(np.float32))
    o32, lse = chronoquant_sdpa_with_lse(cu(g["q1"]), c, scale)
    qs = (g["q1"].astype(np.float64) * float(np.float16(scale))).astype(np.float16).astype(np.float32)
    kk, pk, sk = [npy(x) for x in c._export("k")]
    kv, pv, sv = [npy(x) for x in c._export("v")]
    exact = O.fused_decode(qs[0, :, 0], kk[0], pk[0], sk[0], kv[0], pv[0], sv[0], c.offset, 64, 32, 128)
    # fp32 output of the tensor-core path: P is rounded to fp16 before the PV products
    close(npy(o32)[0, :, 0], exact, atol=3e-4, rtol=3e-3)
    qb = cu(O.bits_to_bf16(g["q1_bf16_bits"])).to(torch.bfloat16)
    ob = chronoquant_sdpa(qb, None, None, c, scale)
    close(npy(ob), O.bits_to_bf16(g["sdpa_fallback_bf16_bits"]))
    c.use_fused = False
    fb = chronoquant_sdpa(cu(g["q1"]), None, None, c, scale)
    close(npy(fb), g["sdpa_fallback"])


def test_dead_zone_and_per_layer_bits(golden_dir):
    from chronoquant_mlx_b200 import ChronoQuantCache
    g = load(golden_dir, "cache_deadzone.npz")
    s = int(g["split"])
    c = build_cache(g["K"], g["V"], [s, g["K"].shape[2] - s], stride_k=8, stride_v=4, delta_bits_k=3,
                    delta_bits_v=4, dead_zone_k=0.1, dead_zone_v=0.2, per_layer_v_bits=[4, 2], layer_idx=1)
    check_state(c, g)
    assert c.nbytes == int(g["nbytes"])
    rk, rv = c.reconstruct_history()
    assert np.array_equal(bits16(npy(rk)), bits16(g["recon_k"]))
    assert np.array_equal(bits16(npy(rv)), bits16(g["recon_v"]))
    c2 = ChronoQuantCache(stride_k=8, stride_v=4)
    c2.state = c.state
    assert c2.offset == int(g["restored_offset"])
    assert c2.nbytes == int(g["restored_nbytes"])
    check_state(c2, g)


# ---------------------------------------------------------------------------- oracle at larger sizes


def oracle_cache(K, V, chunks, **kw):
    c = O.OracleCache(**kw)
    t = 0
    for n in chunks:
        c.update_and_fetch(K[:, :, t:t + n], V[:, :, t:t + n])
        t += n
    return c


def compare_states(gcache, ocache):
    names = ["kf_k", "kf_v", "packed_k", "scales_k", "packed_v", "scales_v"]
    for n, a, b in zip(names, gcache.state, ocache.state):
        a = npy(a)
        assert a.shape == b.shape, n
        assert np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(b).view(np.uint8)), n


@pytest.mark.parametrize("cfg", [
    dict(stride_k=32, stride_v=8, dead_zone_v=0.0),
    dict(stride_k=64, stride_v=32, delta_bits_k=4, delta_bits_v=3, dead_zone_k=0.0, dead_zone_v=0.05),
    dict(stride_k=3, stride_v=5, delta_bits_k=4, delta_bits_v=2, dead_zone_v=0.3),
    dict(stride_k=1, stride_v=2),
])
def test_multi_call_vs_oracle(cfg):
    K, V = O.ar1_kv(2, 3, 700, 128, seed=11)
    chunks = [1, 2, 300, 1, 1, 1, 250, 144]
    g = build_cache(K, V, chunks, page_tokens=None, **cfg)
    o = oracle_cache(K, V, chunks, **cfg)
    compare_states(g, o)
    assert g.nbytes == o.nbytes
    rk, rv = g.reconstruct_history()
    ok, ov = o.reconstruct_history()
    assert np.array_equal(bits16(npy(rk)), bits16(ok))
    assert np.array_equal(bits16(npy(rv)), bits16(ov))


@pytest.mark.parametrize("D", [64, 72, 256])
def test_other_head_dims(D):
    from chronoquant_mlx_b200 import chronoquant_sdpa
    K, V = O.ar1_kv(1, 2, 300, D, seed=D)
    g = build_cache(K, V, [150, 1, 149], stride_k=32, stride_v=8)
    o = oracle_cache(K, V, [150, 1, 149], stride_k=32, stride_v=8)
    compare_states(g, o)
    q = (np.random.default_rng(0).standard_normal((1, 4, 1, D)) / math.sqrt(D)).astype(np.float16)
    scale = 1.0 / math.sqrt(D)
    out = chronoquant_sdpa(cu(q), None, None, g, scale)
    qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    k32, v32 = o.reconstruct_history_f32()
    close(npy(out), O.exact_sdpa(qs, k32, v32, False))


def test_bf16_tokens_vs_oracle():
    K, V = O.ar1_kv(1, 2, 200, 128, seed=5)
    Kb = O.round_bf16(K.astype(np.float32) * 3.0)
    Vb = O.round_bf16(V.astype(np.float32))
    g = build_cache(Kb, Vb, [77, 123], dtype=torch.bfloat16, stride_k=32, stride_v=8)
    o = O.OracleCache(stride_k=32, stride_v=8, dtype="bf16")
    o.update_and_fetch(Kb[:, :, :77], Vb[:, :, :77])
    o.update_and_fetch(Kb[:, :, 77:], Vb[:, :, 77:])
    compare_states(g, o)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("cfg", [
    dict(stride_k=32, stride_v=8, dead_zone_v=0.0),
    dict(stride_k=64, stride_v=32, delta_bits_v=3, dead_zone_v=0.05),
    dict(stride_k=16, stride_v=4, delta_bits_k=2, delta_bits_v=2, dead_zone_k=0.2),
])
def test_bulk_append_matches_token_appends(dtype, cfg):
    """A multi-token append (head_dim 128: the 8-token-block kernel, codes from
    a reciprocal with an exact FMA check near rounding boundaries) against the
    same tokens appended one call each (the one-token kernel, a division per
    value) and against the oracle, bit for bit.  Token magnitudes span the
    dtype's range (fp16: subnormal to 1e3 scales; bf16: down to 1e-38, where
    1/scale overflows and the division is taken)."""
    rng = np.random.default_rng(17 if dtype == "f16" else 18)
    B, H, T, D = 1, 2, 320, 128
    K, V = O.ar1_kv(B, H, T, D, seed=3)
    lo, hi = (-7.0, 3.0) if dtype == "f16" else (-38.0, 3.0)
    mag = 10.0 ** rng.uniform(lo, hi, size=(B, H, T, 1))
    K = K.astype(np.float64) * mag
    V = V.astype(np.float64) * mag[:, :, ::-1]
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    if dtype == "f16":
        K, V = K.astype(np.float16), V.astype(np.float16)
    else:
        K, V = O.round_bf16(K.astype(np.float32)), O.round_bf16(V.astype(np.float32))
    bulk = build_cache(K, V, [5, 200, 115], dtype=tdt, **cfg)
    single = build_cache(K, V, [1] * T, dtype=tdt, **cfg)
    for a, b in zip(bulk.state, single.state):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    o = O.OracleCache(dtype=dtype, **cfg)
    for t0, n in ((0, 5), (5, 200), (205, 115)):
        o.update_and_fetch(K[:, :, t0:t0 + n], V[:, :, t0:t0 + n])
    compare_states(bulk, o)


@pytest.mark.parametrize("B,Hkv,Hq,T,cfg", [
    (1, 8, 32, 4096, dict(stride_k=32, stride_v=8, dead_zone_v=0.0)),
    (3, 2, 16, 1000, dict(stride_k=64, stride_v=32, delta_bits_v=3)),
    (2, 4, 4, 777, dict(stride_k=32, stride_v=8)),
    (2, 2, 32, 513, dict(stride_k=16, stride_v=16)),
])
def test_decode_attention_vs_exact(B, Hkv, Hq, T, cfg):
    from chronoquant_mlx_b200 import chronoquant_sdpa
    from chronoquant_mlx_b200.attention import chronoquant_sdpa_with_lse
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=T)
    g = build_cache(K, V, [T - 1, 1], **cfg)
    o = oracle_cache(K, V, [T - 1, 1], **cfg)
    compare_states(g, o)
    scale = 1.0 / math.sqrt(128)
    q = (np.random.default_rng(T).standard_normal((B, Hq, 1, 128)) / math.sqrt(128)).astype(np.float32)
    qb = O.round_bf16(q)
    qs = O.round_bf16(qb.astype(np.float64) * float(O.round_bf16(np.float32(scale))))
    k32, v32 = o.reconstruct_history_f32()
    exact = O.exact_sdpa(qs, k32, v32, False)
    out = chronoquant_sdpa(cu(qb, torch.bfloat16), None, None, g, scale)
    close(npy(out), exact)
    o32, lse = chronoquant_sdpa_with_lse(cu(qb, torch.bfloat16), g, scale)
    close(npy(o32), exact, atol=3e-4, rtol=3e-3)
    # the reference's fallback for B>1 (fp16 reconstruction, fp32-promoted scores for bf16 queries)
    fk, fv = o.reconstruct_history()
    fb = O.fallback_sdpa(qb, "bf16", fk, fv, scale, None)
    close(npy(out), fb)


def test_prefill_chunk_causal_vs_exact():
    from chronoquant_mlx_b200 import chronoquant_sdpa
    K, V = O.ar1_kv(1, 2, 640, 128, seed=9)
    g = build_cache(K, V, [512, 128], stride_k=32, stride_v=8)
    o = oracle_cache(K, V, [512, 128], stride_k=32, stride_v=8)
    q = (np.random.default_rng(1).standard_normal((1, 8, 128, 128)) / math.sqrt(128)).astype(np.float16)
    scale = 1.0 / math.sqrt(128)
    out = chronoquant_sdpa(cu(q), None, None, g, scale, mask=g.make_mask(128))
    qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    k32, v32 = o.reconstruct_history_f32()
    close(npy(out), O.exact_sdpa(qs, k32, v32, True))
    fk, fv = o.reconstruct_history()
    close(npy(out), O.fallback_sdpa(q, "f16", fk, fv, scale, "causal"))


def assert_ties_match(dev_state, ora_state, tie_sites, D=128):
    """The quotients the oracle found exactly halfway between two integers
    (codec.py:50-51 rounds them half to even): check that the device's codes
    equal the oracle's at every one of them.  Returns the tie count per
    component ("k", "v").  States are the reference layout [kf_k, kf_v,
    packed_k, scales_k, packed_v, scales_v] of one (sequence, kv-head)."""
    counts = {}
    for comp, idx in (("k", 2), ("v", 4)):
        mask = np.concatenate(tie_sites[comp], axis=2)
        dev = O.unpack_int4(np.ascontiguousarray(dev_state[idx]), D)
        ora = O.unpack_int4(np.ascontiguousarray(ora_state[idx]), D)
        assert mask.shape == dev.shape == ora.shape
        assert np.array_equal(dev[mask], ora[mask])
        counts[comp] = int(mask.sum())
    return counts


def test_full_size_config2_properties():
    """bench config 2 sizes (B8 Hkv8 Hq32 T16384): encode of two rows
    bit-exact against the oracle, export->import idempotent, decode of two
    heads against exact attention."""
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    B, H, T, D = 8, 8, 16384, 128
    K, V = O.ar1_kv_fast(B, H, T, D, seed=0)
    c = ChronoQuantCache(stride_k=32, stride_v=8, dead_zone_v=0.0, max_tokens=T + 64)
    c.update_and_fetch(cu(K[:, :, :T - 1]), cu(V[:, :, :T - 1]))
    c.update_and_fetch(cu(K[:, :, T - 1:]), cu(V[:, :, T - 1:]))
    st = c.state
    for (b, h) in ((0, 0), (7, 5)):
        o = O.OracleCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
        sites = {}
        o.update_and_fetch(K[b:b + 1, h:h + 1], V[b:b + 1, h:h + 1], tie_sites=sites)
        dev = [npy(a[b:b + 1, h:h + 1]) for a in st]
        for a, r in zip(dev, o.state):
            assert np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(r).view(np.uint8))
        ties = assert_ties_match(dev, o.state, sites)
        print(f"config 2 unit ({b},{h}): {ties['k']} K and {ties['v']} V halfway quotients, all matched")
    c2 = ChronoQuantCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
    c2.state = st
    for a, b in zip(st, c2.state):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    q = (np.random.default_rng(2).standard_normal((B, 32, 1, D)) / math.sqrt(D)).astype(np.float16)
    scale = 1.0 / math.sqrt(D)
    out = npy(chronoquant_sdpa(cu(q), None, None, c, scale))
    qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    for (b, h) in ((0, 0), (7, 5)):
        o = O.OracleCache(stride_k=32, stride_v=8, dead_zone_v=0.0)
        o.update_and_fetch(K[b:b + 1, h:h + 1], V[b:b + 1, h:h + 1])
        k32, v32 = o.reconstruct_history_f32()
        ex = O.exact_sdpa(qs[b:b + 1, 4 * h:4 * h + 4], k32, v32, False)
        close(out[b:b + 1, 4 * h:4 * h + 4], ex)


def test_sequence_shard_merge():
    """Attention over two key shards merged by log-sum-exp equals attention
    over the whole sequence."""
    import ctypes
    from chronoquant_mlx_b200 import _lib
    from chronoquant_mlx_b200.attention import chronoquant_sdpa_with_lse
    K, V = O.ar1_kv(2, 2, 1024, 128, seed=4)
    full = build_cache(K, V, [1024], stride_k=32, stride_v=8)
    a = build_cache(K[:, :, :512], V[:, :, :512], [512], stride_k=32, stride_v=8)
    b = build_cache(K[:, :, 512:], V[:, :, 512:], [512], stride_k=32, stride_v=8)
    q = cu((np.random.default_rng(8).standard_normal((2, 8, 1, 128)) / math.sqrt(128)).astype(np.float16))
    scale = 1.0 / math.sqrt(128)
    of, lf = chronoquant_sdpa_with_lse(q, full, scale)
    oa, la = chronoquant_sdpa_with_lse(q, a, scale)
    ob, lb = chronoquant_sdpa_with_lse(q, b, scale)
    lse = torch.stack([la, lb]).contiguous()
    o = torch.stack([oa, ob]).contiguous()
    out = torch.empty_like(of)
    rows = of.numel() // 128
    _lib.check(_lib.lib().cq_lse_merge(lse.data_ptr(), o.data_ptr(), 2, rows, 128, out.data_ptr(), _lib.CQ_F32,
                                       torch.cuda.current_stream().cuda_stream))
    # the same partials packed one buffer per part ([outputs | lse], as one all-gather delivers them)
    packed = torch.cat([o.reshape(2, rows * 128), lse.reshape(2, rows)], dim=1).contiguous()
    out_p = torch.empty_like(of)
    _lib.check(_lib.lib().cq_lse_merge_packed(packed.data_ptr(), 2, rows, 128, out_p.data_ptr(), _lib.CQ_F32,
                                              torch.cuda.current_stream().cuda_stream))
    assert torch.equal(out_p, out)
    # shard b re-anchors at its first token, so compare against the exact union of both shards' decodes
    oa_ = O.OracleCache(stride_k=32, stride_v=8)
    oa_.update_and_fetch(K[:, :, :512], V[:, :, :512])
    ob_ = O.OracleCache(stride_k=32, stride_v=8)
    ob_.update_and_fetch(K[:, :, 512:], V[:, :, 512:])
    ka, va = oa_.reconstruct_history_f32()
    kb, vb = ob_.reconstruct_history_f32()
    qs = (npy(q).astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    ex = O.exact_sdpa(qs, np.concatenate([ka, kb], 2), np.concatenate([va, vb], 2), False)
    close(npy(out), ex, atol=1e-4, rtol=1e-3)
    # a 512-token shard boundary is a multiple of both strides: same anchors as the full cache
    close(npy(out), npy(of), atol=1e-5, rtol=1e-4)


def test_errors():
    from chronoquant_mlx_b200 import ChronoQuantCache
    c = ChronoQuantCache()
    with pytest.raises(ValueError):
        c.update_and_fetch(torch.zeros(1, 2, 3, 128, dtype=torch.float16),
                           torch.zeros(1, 2, 3, 128, dtype=torch.float16))
    c.update_and_fetch(torch.zeros(1, 2, 3, 128, dtype=torch.float16, device="cuda"),
                       torch.zeros(1, 2, 3, 128, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError, match="head_dim changed"):
        c.update_and_fetch(torch.zeros(1, 2, 3, 64, dtype=torch.float16, device="cuda"),
                           torch.zeros(1, 2, 3, 64, dtype=torch.float16, device="cuda"))


def test_no_device_timeouts_recorded():
    import ctypes
    from chronoquant_mlx_b200 import _lib
    code = ctypes.c_int(-1)
    _lib.check(_lib.lib().cq_device_error(ctypes.byref(code), 1))
    assert code.value == 0


@pytest.mark.parametrize("T", [1, 2, 15, 16, 17, 255, 256, 257, 1000])
def test_decode_fast_vs_generic_small_T(T):
    """Decode through the fast kernel (paged cache) and through the general
    kernel (the reconstruct path, use_fused=False) on the same cache."""
    from chronoquant_mlx_b200 import chronoquant_sdpa
    K, V = O.ar1_kv(2, 2, T, 128, seed=T + 100)
    g = build_cache(K, V, [T], stride_k=32, stride_v=8)
    o = oracle_cache(K, V, [T], stride_k=32, stride_v=8)
    q = (np.random.default_rng(T).standard_normal((2, 8, 1, 128)) / math.sqrt(128)).astype(np.float16)
    scale = 1.0 / math.sqrt(128)
    out = chronoquant_sdpa(cu(q), None, None, g, scale)
    qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    k32, v32 = o.reconstruct_history_f32()
    close(npy(out), O.exact_sdpa(qs, k32, v32, False))
    g.use_fused = False
    out2 = chronoquant_sdpa(cu(q), None, None, g, scale)
    close(npy(out2), npy(out))


def test_full_size_config3_properties():
    """bench config 3 sizes (B16 Hkv8 Hq32 T32768, Full-Throttle V3: strides
    64/32, 4/3 bits, dead zones 0/0.05, AR(1) K/V with rho 0.97/0.85): the
    state of three sampled (sequence, kv-head) units bit-exact against the
    oracle (halfway quotients counted and matched), decode of their query
    heads on the sm_100a kernel against exact float64 attention and against
    the reference's fp16 fallback (B > 1), within 2e-3 / 1e-2."""
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    B, H, T, D = 16, 8, 32768, 128
    kw = dict(stride_k=64, stride_v=32, delta_bits_k=4, delta_bits_v=3, dead_zone_k=0.0, dead_zone_v=0.05)
    K, V = O.ar1_kv_fast(B, H, T, D, rho_k=0.97, rho_v=0.85, seed=3)
    c = ChronoQuantCache(max_tokens=T + 64, **kw)
    for t in range(0, T, 8192):  # prefill in chunks, as a serving loop would
        c.update_and_fetch(cu(K[:, :, t:t + 8192]), cu(V[:, :, t:t + 8192]))
    st = c.state
    q = (np.random.default_rng(4).standard_normal((B, 32, 1, D)) / math.sqrt(D)).astype(np.float32)
    qb = O.round_bf16(q)
    scale = 1.0 / math.sqrt(D)
    out = npy(chronoquant_sdpa(cu(qb, torch.bfloat16), None, None, c, scale))
    qs = O.round_bf16(qb.astype(np.float64) * float(O.round_bf16(np.float32(scale))))
    for (b, h) in ((0, 0), (9, 3), (15, 7)):
        o = O.OracleCache(**kw)
        sites = {}
        for t in range(0, T, 8192):
            o.update_and_fetch(K[b:b + 1, h:h + 1, t:t + 8192], V[b:b + 1, h:h + 1, t:t + 8192], tie_sites=sites)
        dev = [npy(a[b:b + 1, h:h + 1]) for a in st]
        for a, r in zip(dev, o.state):
            assert np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(r).view(np.uint8))
        ties = assert_ties_match(dev, o.state, sites)
        print(f"config 3 unit ({b},{h}): {ties['k']} K and {ties['v']} V halfway quotients, all matched")
        k32, v32 = o.reconstruct_history_f32()
        rows = slice(4 * h, 4 * h + 4)
        close(out[b:b + 1, rows], O.exact_sdpa(qs[b:b + 1, rows], k32, v32, False))
        fk, fv = o.reconstruct_history()
        close(out[b:b + 1, rows], O.fallback_sdpa(qb[b:b + 1, rows], "bf16", fk, fv, scale, None))
