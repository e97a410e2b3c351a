"""Query chunks (chunked prefill) on the tensor-core path, against the oracle.

The reference answers q_len > 1 with its fallback (attention.py:61-74): fp16
reconstruction of the history, q * scale in the query dtype, scores, causal
mask anchored at the end of the keys, softmax, weights @ V.  Each case builds
the cache as the reference's flow does (context, then the chunk appended by
update_and_fetch) and compares ``chronoquant_sdpa`` with

* ``O.fallback_sdpa`` on the oracle's fp16 reconstruction (the reference
  path): max-abs 2e-3 / relative 1e-2;
* exact float64 attention on the same fp16 values: max-abs 1e-3 / relative
  5e-3 (the kernel rounds only the softmax weights, to fp16).

The full-size case (bench config 4: 65536 cached tokens + a 2048-token
chunk, 32 query heads over 8 kv-heads) checks sampled rows against exact
float64 attention on the device's fp16 reconstruction, which other tests pin
bit-exact to the oracle."""

import math

import numpy as np
import pytest
import torch

from oracle import cq_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
EX_ATOL, EX_RTOL = 1e-3, 5e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import chronoquant_mlx_b200._lib as L
    L.lib()


def close(out, ref, atol, rtol):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(out - ref)
    ok = err <= atol + rtol * np.abs(ref)
    assert ok.all(), f"max abs err {err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}"


def npy(t):
    return t.detach().float().cpu().numpy()


def scaled_q(q, q_dtype, scale):
    """q * scale rounded to the query dtype, as the reference's q_scaled."""
    if q_dtype == "f16":
        return (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    return O.round_bf16(q.astype(np.float64) * float(O.round_bf16(np.float32(scale))))


CASES = [
    # B, Hkv, Hq, T, q_len, stride_k, stride_v, bits_v, dz_v, q dtype, causal
    (1, 2, 8, 1000, 100, 32, 8, 4, 0.0, "bf16", True),      # GQA 4, ragged tiles
    (2, 2, 2, 777, 200, 32, 8, 4, 0.05, "f16", False),      # GQA 1, mask None
    (1, 2, 16, 300, 40, 32, 8, 4, 0.05, "bf16", True),      # GQA 8
    (1, 1, 16, 513, 16, 64, 32, 3, 0.05, "f16", True),      # GQA 16, FT-V3, shortest chunk
    (2, 4, 16, 2100, 300, 64, 32, 3, 0.05, "bf16", True),   # FT-V3, several key tiles
    (1, 2, 8, 256, 256, 32, 8, 4, 0.0, "f16", True),        # chunk = whole cache (first prefill)
    (1, 2, 8, 1024, 1024, 32, 8, 4, 0.0, "bf16", True),     # key-range splits, some ranges empty
    (2, 2, 8, 3000, 64, 32, 8, 4, 0.0, "f16", False),       # key-range splits, mask None
]


@pytest.mark.parametrize("B,Hkv,Hq,T,q_len,sk,sv,bv,dzv,qdt,causal", CASES)
def test_prefill_chunk_vs_oracle(B, Hkv, Hq, T, q_len, sk, sv, bv, dzv, qdt, causal):
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=T + q_len)
    kw = dict(stride_k=sk, stride_v=sv, delta_bits_k=4, delta_bits_v=bv, dead_zone_k=0.0, dead_zone_v=dzv)
    cache = ChronoQuantCache(**kw)
    oc = O.OracleCache(**kw)
    for t0, n in ((0, T - q_len), (T - q_len, q_len)):
        if n:
            cache.update_and_fetch(torch.from_numpy(K[:, :, t0:t0 + n]).cuda(),
                                   torch.from_numpy(V[:, :, t0:t0 + n]).cuda())
            oc.update_and_fetch(K[:, :, t0:t0 + n], V[:, :, t0:t0 + n])
    rng = np.random.default_rng(q_len)
    q = rng.standard_normal((B, Hq, q_len, 128)) / math.sqrt(128)
    if qdt == "f16":
        q = q.astype(np.float16)
        qt = torch.from_numpy(q).cuda()
    else:
        q = O.round_bf16(q.astype(np.float32))
        qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    mask = "causal" if causal else None
    out = chronoquant_sdpa(qt, None, None, cache, scale, mask=mask)
    assert out.dtype == qt.dtype and out.shape == (B, Hq, q_len, 128)
    fk, fv = oc.reconstruct_history()
    close(npy(out), O.fallback_sdpa(q, qdt, fk, fv, scale, mask), ATOL, RTOL)
    close(npy(out), O.exact_sdpa(scaled_q(q, qdt, scale), fk, fv, causal), EX_ATOL, EX_RTOL)


def test_prefill_lse_and_strided_queries():
    """fp32 output and log-sum-exp through chronoquant_sdpa_with_lse, queries
    given as a transposed [B, q_len, Hq, D] view (non-contiguous heads)."""
    from chronoquant_mlx_b200 import ChronoQuantCache
    from chronoquant_mlx_b200.attention import chronoquant_sdpa_with_lse
    B, Hkv, Hq, T, q_len = 2, 2, 8, 900, 64
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=5)
    cache = ChronoQuantCache(stride_k=32, stride_v=8)
    oc = O.OracleCache(stride_k=32, stride_v=8)
    cache.update_and_fetch(torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda())
    oc.update_and_fetch(K, V)
    q = (np.random.default_rng(3).standard_normal((B, q_len, Hq, 128)) / math.sqrt(128)).astype(np.float16)
    qt = torch.from_numpy(q).cuda().transpose(1, 2)  # [B, Hq, q_len, D], strides (.., D, Hq*D, 1)
    scale = 1.0 / math.sqrt(128)
    out, lse = chronoquant_sdpa_with_lse(qt, cache, scale)
    qs = scaled_q(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), "f16", scale)
    fk, fv = oc.reconstruct_history()
    close(npy(out), O.exact_sdpa(qs, fk, fv, True), EX_ATOL, EX_RTOL)
    # natural-log log-sum-exp of the causal scores
    s = np.einsum("bgrqd,bgtd->bgrqt", qs.astype(np.float64).reshape(B, Hkv, Hq // Hkv, q_len, 128),
                  fk.astype(np.float64))
    s = np.where(O.causal_mask(q_len, T), s, -np.inf)
    mx = s.max(-1, keepdims=True)
    ref = (mx[..., 0] + np.log(np.exp(s - mx).sum(-1))).reshape(B, Hq, q_len)
    close(npy(lse), ref, 1e-3, 1e-4)


def test_prefill_config4_sampled_rows():
    """bench config 4: B1 Hq32 Hkv8 D128, 65536 compressed tokens then a
    2048-token chunk (Standard strides), causal.  For the kv-heads of the
    sampled rows (query-tile edges, first/last tokens, every GQA position) the
    oracle encodes the same tokens on the CPU; its fp16 reconstruction
    (cache.py:131-160, the reference's fallback input) must equal the
    device's bit for bit, and the sampled rows must match exact float64
    attention over the oracle's reconstruction."""
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    B, Hkv, Hq, ctx, chunk = 1, 8, 32, 65536, 2048
    T = ctx + chunk
    K, V = O.ar1_kv_fast(B, Hkv, T, 128, seed=4)
    cache = ChronoQuantCache(stride_k=32, stride_v=8)
    cache.update_and_fetch(torch.from_numpy(K[:, :, :ctx]).cuda(), torch.from_numpy(V[:, :, :ctx]).cuda())
    cache.update_and_fetch(torch.from_numpy(K[:, :, ctx:]).cuda(), torch.from_numpy(V[:, :, ctx:]).cuda())
    q = O.round_bf16((np.random.default_rng(7).standard_normal((B, Hq, chunk, 128)) / math.sqrt(128))
                     .astype(np.float32))
    scale = 1.0 / math.sqrt(128)
    out = npy(chronoquant_sdpa(torch.from_numpy(q).cuda().to(torch.bfloat16), None, None, cache, scale,
                               mask="causal"))
    assert np.isfinite(out).all()
    dk, dv = (npy(t) for t in cache.reconstruct_history())
    qs = scaled_q(q, "bf16", scale).astype(np.float64)
    toks = [0, 1, 31, 32, 63, 1000, 2015, 2016, 2047]
    heads = (0, 5, 10, 15, 20, 27, 31)
    recon = {}
    for kh in sorted({hq // (Hq // Hkv) for hq in heads}):
        o = O.OracleCache(stride_k=32, stride_v=8)
        o.update_and_fetch(K[:, kh:kh + 1, :ctx], V[:, kh:kh + 1, :ctx])
        o.update_and_fetch(K[:, kh:kh + 1, ctx:], V[:, kh:kh + 1, ctx:])
        fk, fv = o.reconstruct_history()
        assert np.array_equal(dk[:, kh:kh + 1].astype(np.float16).view(np.uint16), fk.view(np.uint16))
        assert np.array_equal(dv[:, kh:kh + 1].astype(np.float16).view(np.uint16), fv.view(np.uint16))
        recon[kh] = (fk[0, 0].astype(np.float64), fv[0, 0].astype(np.float64))
    del K, V
    for hq in heads:
        fk, fv = recon[hq // (Hq // Hkv)]
        for i in toks:
            lim = ctx + i + 1
            s = fk[:lim] @ qs[0, hq, i]
            p = np.exp(s - s.max())
            ref = (p @ fv[:lim]) / p.sum()
            close(out[0, hq, i], O.round_bf16(ref.astype(np.float32)), ATOL, RTOL)
