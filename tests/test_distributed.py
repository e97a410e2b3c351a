"""Sequence-split attention (one long sequence over several ranks): the shard
layout, the gloo exchange of partials on world-size-2 CPU ranks, failure
detection when a rank leaves, and the CUDA merge on one GPU.

Bars: shard bounds aligned to lcm(stride_k, stride_v) and covering [0, T);
each shard's compressed state bit-identical to the slice of the unsplit
cache; merged partials within 1e-12 (float64 protocol test) / max-abs 2e-3,
relative 1e-2 (CUDA merge) of unsplit attention."""

import math
import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from oracle import cq_oracle as O
from chronoquant_mlx_b200.distributed import merge_partials, shard_bounds

import _dist_workers as W


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("T,world,sk,sv", [(1000, 2, 32, 8), (4096, 8, 64, 32), (5, 4, 4, 2), (0, 3, 32, 8),
                                           (65536 + 2048, 8, 32, 8)])
def test_shard_bounds(T, world, sk, sv):
    b = shard_bounds(T, world, sk, sv)
    align = sk * sv // math.gcd(sk, sv)
    assert len(b) == world and b[0][0] == 0 and b[-1][1] == T
    for (lo, hi), (lo2, _) in zip(b, b[1:]):
        assert hi == lo2
    for lo, hi in b:
        assert lo <= hi and (lo % align == 0 or lo == T)


def test_shards_are_slices_of_the_unsplit_cache():
    """Each shard starts on an I-frame of both components, so its encoded state
    is exactly the matching slice of the unsplit cache's state."""
    K, V = O.ar1_kv(1, 2, 300, 128, seed=2)
    full = O.OracleCache(stride_k=32, stride_v=8)
    full.update_and_fetch(K, V)
    parts = []
    for lo, hi in shard_bounds(300, 3, 32, 8):
        c = O.OracleCache(stride_k=32, stride_v=8)
        c.update_and_fetch(K[:, :, lo:hi], V[:, :, lo:hi])
        parts.append(c.state)
    for i, ref in enumerate(full.state):
        cat = np.concatenate([p[i] for p in parts], axis=2)
        assert cat.shape == ref.shape, i
        assert np.array_equal(np.ascontiguousarray(cat).view(np.uint8), np.ascontiguousarray(ref).view(np.uint8)), i


def _run(target, args_for_rank, world, timeout=120, reporting=None):
    """Start `world` spawned ranks; collect one queue message from each
    reporting rank; return (messages by rank, exit codes)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=args_for_rank(r) + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    n = world if reporting is None else len(reporting)
    out = [q.get(timeout=timeout) for _ in range(n)]
    for p in procs:
        p.join(timeout=timeout)
    return sorted(out, key=lambda x: x[0]), [p.exitcode for p in procs]


@pytest.mark.parametrize("q_len", [1, 48])
def test_gloo_exchange_and_merge(q_len):
    """World size 2 on CPU: every rank gathers both partials in rank order, and
    the log-sum-exp merge equals attention over the whole sequence."""
    B, Hkv, Hq, T, sk, sv = 1, 2, 8, 640, 32, 8
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=11)
    q = (np.random.default_rng(1).standard_normal((B, Hq, q_len, 128)) / math.sqrt(128)).astype(np.float16)
    qs = (q.astype(np.float64) * float(np.float16(1 / math.sqrt(128)))).astype(np.float16)
    port = _free_port()
    res, codes = _run(W.shard_worker, lambda r: (r, 2, port, K, V, qs, sk, sv), 2)
    assert codes == [0, 0]
    for rank, o_all, lse_all, err in res:
        assert err is None, err
        assert o_all.shape == (2, B, Hq, q_len, 128) and lse_all.shape == (2, B, Hq, q_len)
        M = lse_all.max(0)
        w = np.exp(lse_all - M)
        merged = (w[..., None] * o_all).sum(0) / w.sum(0)[..., None]
        full = O.OracleCache(stride_k=sk, stride_v=sv)
        full.update_and_fetch(K, V)
        k32, v32 = full.reconstruct_history_f32()
        ref = O.exact_sdpa(qs, k32, v32, causal=True)
        assert np.abs(merged - ref).max() < 1e-12


@pytest.mark.parametrize("T,world,q_len", [(64, 3, 8), (100, 2, 48)])
def test_gloo_short_tail_shard_raises_on_every_rank(T, world, q_len):
    """A query chunk longer than the tail shard (T=64 over 3 ranks leaves the
    tail empty; T=100 over 2 leaves 4 tokens for 48 queries) would put some of
    the chunk's own tokens in an unmasked shard: every rank raises instead."""
    from chronoquant_mlx_b200.distributed import shard_bounds
    tail = shard_bounds(T, world, 32, 8)[-1]
    assert tail[1] - tail[0] < q_len
    port = _free_port()
    res, codes = _run(W.short_tail_worker, lambda r: (r, world, port, T, q_len, 32, 8), world)
    assert codes == [0] * world
    for rank, msg, n in res:
        assert msg.startswith("raised:") and "tail shard" in msg, (rank, msg)


def test_gloo_rank_failure_is_detected():
    """A rank that leaves before the exchange (a host-side failure: no GPU is
    involved) makes the other rank's collective raise instead of hanging."""
    port = _free_port()
    res, codes = _run(W.failing_worker, lambda r: (r, 2, port), 2, timeout=90, reporting=[0])
    assert codes[1] == 3  # rank 1 left
    assert res[0][0] == 0 and res[0][1].startswith("error"), res[0][1]


def test_merge_partials_has_no_cpu_fallback():
    with pytest.raises(ValueError, match="CUDA"):
        merge_partials(torch.zeros(2, 1, 4, 1, 128), torch.zeros(2, 1, 4, 1))


@pytest.mark.gpu
@pytest.mark.parametrize("q_len", [1, 64])
def test_shard_partials_merge_on_gpu(q_len):
    """Two shards emulated on one GPU: local_partials of each (the tail causal
    for a chunk), merged by cq_lse_merge, against exact attention over the
    whole sequence."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache
    from chronoquant_mlx_b200.distributed import local_partials
    B, Hkv, Hq, T = 2, 2, 8, 1536
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=21)
    q = (np.random.default_rng(2).standard_normal((B, Hq, q_len, 128)) / math.sqrt(128)).astype(np.float16)
    scale = 1 / math.sqrt(128)
    os_, ls_ = [], []
    bounds = shard_bounds(T, 2, 32, 8)
    for i, (lo, hi) in enumerate(bounds):
        c = ChronoQuantCache(stride_k=32, stride_v=8)
        c.update_and_fetch(torch.from_numpy(K[:, :, lo:hi]).cuda(), torch.from_numpy(V[:, :, lo:hi]).cuda())
        o, lse = local_partials(torch.from_numpy(q).cuda(), c, scale, tail=i == len(bounds) - 1)
        os_.append(o)
        ls_.append(lse)
    out = merge_partials(torch.stack(os_), torch.stack(ls_))
    full = O.OracleCache(stride_k=32, stride_v=8)
    full.update_and_fetch(K, V)
    k32, v32 = full.reconstruct_history_f32()
    qs = (q.astype(np.float64) * float(np.float16(scale))).astype(np.float16)
    ref = O.exact_sdpa(qs, k32, v32, causal=True)
    err = np.abs(out.cpu().numpy() - ref)
    assert (err <= 2e-3 + 1e-2 * np.abs(ref)).all(), err.max()


@pytest.mark.gpu
@pytest.mark.parametrize("q_len", [1, 64])
def test_nccl_sequence_split_two_gpus(q_len):
    """Two ranks on two GPUs: each holds half the sequence, the partials cross
    NVLink in one NCCL all-gather, and every rank's merged output matches
    exact attention over the whole sequence."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    B, Hkv, Hq, T, sk, sv = 2, 2, 8, 2048, 32, 8
    K, V = O.ar1_kv(B, Hkv, T, 128, seed=31)
    q = (np.random.default_rng(4).standard_normal((B, Hq, q_len, 128)) / math.sqrt(128)).astype(np.float16)
    port = _free_port()
    res, codes = _run(W.nccl_worker, lambda r: (r, 2, port, K, V, q, sk, sv), 2, timeout=180)
    full = O.OracleCache(stride_k=sk, stride_v=sv)
    full.update_and_fetch(K, V)
    k32, v32 = full.reconstruct_history_f32()
    qs = (q.astype(np.float64) * float(np.float16(1 / math.sqrt(128)))).astype(np.float16)
    ref = O.exact_sdpa(qs, k32, v32, causal=True)
    for rank, out, err in res:
        assert err is None, err
        e = np.abs(out - ref)
        assert (e <= 2e-3 + 1e-2 * np.abs(ref)).all(), (rank, e.max())
    assert codes == [0, 0]


@pytest.mark.parametrize("n_seq", [1, 2, 4])
def test_mesh_groups(n_seq):
    """mesh_groups on 4 gloo ranks: rank r = s * tp + p sits in the
    tensor-parallel group of its s and the sequence group of its p, and a
    collective over the sequence group sums exactly those ranks."""
    import multiprocessing as mp
    import socket
    import _dist_workers as W
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
    sk.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=W.mesh_groups_worker, args=(r, 4, port, n_seq, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(4)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    tp = 4 // n_seq
    for rank, tp_ranks, seq_ranks, seq_sum, err in res:
        assert err is None, err
        s, p = divmod(rank, tp)
        assert tp_ranks == (None if tp == 1 else [s * tp + i for i in range(tp)])
        want_seq = [i * tp + p for i in range(n_seq)]
        assert seq_ranks == (None if n_seq == 1 else want_seq)
        assert seq_sum == (None if n_seq == 1 else sum(want_seq))
