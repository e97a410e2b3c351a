"""Process bodies for the gloo (CPU) tests of the sequence-split protocol.

Each rank holds one shard of a sequence (``shard_bounds``), computes its exact
partial attention with the oracle (float64 numpy: the test's checker), and
exchanges partials with ``exchange_partials`` over a gloo process group.
Results go back through a multiprocessing queue."""

import ctypes
import datetime
import math
import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import cq_oracle as O


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def exact_partial(q_scaled, k, v, causal):
    """(o [B,Hq,Tq,D], lse [B,Hq,Tq]) of float64 attention of q over one
    shard's decoded k/v; causal anchors the mask at the end of the shard."""
    B, Hq, Tq, D = q_scaled.shape
    Hkv, T = k.shape[1], k.shape[2]
    if T == 0:
        return np.zeros((B, Hq, Tq, D)), np.full((B, Hq, Tq), -np.inf)
    qg = q_scaled.astype(np.float64).reshape(B, Hkv, Hq // Hkv, Tq, D)
    s = np.einsum("bgrqd,bgtd->bgrqt", qg, k.astype(np.float64))
    if causal and Tq > 1:
        s = np.where(O.causal_mask(Tq, T), s, -np.inf)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    lsum = p.sum(-1)
    o = np.einsum("bgrqt,bgtd->bgrqd", p, v.astype(np.float64)) / lsum[..., None]
    return o.reshape(B, Hq, Tq, D), (m[..., 0] + np.log(lsum)).reshape(B, Hq, Tq)


def shard_worker(rank, world, port, K, V, q_scaled, stride_k, stride_v, queue):
    """Encode this rank's shard with the oracle, take the exact partial, all-gather."""
    from chronoquant_mlx_b200.distributed import exchange_partials, shard_bounds
    try:
        _init(rank, world, port, 30)
        T = K.shape[2]
        lo, hi = shard_bounds(T, world, stride_k, stride_v)[rank]
        c = O.OracleCache(stride_k=stride_k, stride_v=stride_v)
        if hi > lo:
            c.update_and_fetch(K[:, :, lo:hi], V[:, :, lo:hi])
            k, v = c.reconstruct_history_f32()
        else:
            k = np.zeros(K.shape[:2] + (0, K.shape[3]))
            v = k
        o, lse = exact_partial(q_scaled, k, v, causal=rank == world - 1)
        o_all, lse_all = exchange_partials(torch.from_numpy(o), torch.from_numpy(lse))
        queue.put((rank, o_all.numpy(), lse_all.numpy(), None))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        queue.put((rank, None, None, repr(e)))


def failing_worker(rank, world, port, queue):
    """Rank 1 fails before the exchange (a host-side fault); rank 0 must see
    an error from its collective within the process-group timeout."""
    from chronoquant_mlx_b200.distributed import exchange_partials
    _init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)  # leaves without joining the collective (exit code 3)
    try:
        exchange_partials(torch.zeros(1, 2, 1, 8), torch.zeros(1, 2, 1))
        queue.put((rank, "no error"))
    except Exception as e:
        queue.put((rank, "error: " + type(e).__name__))


def nccl_worker(rank, world, port, K, V, q, stride_k, stride_v, queue):
    """One GPU per rank: encode this rank's shard with the CUDA path, run
    sequence_parallel_attention (NCCL all-gather over NVLink + cq_lse_merge)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from chronoquant_mlx_b200 import ChronoQuantCache
        from chronoquant_mlx_b200.distributed import sequence_parallel_attention, shard_bounds
        lo, hi = shard_bounds(K.shape[2], world, stride_k, stride_v)[rank]
        c = ChronoQuantCache(stride_k=stride_k, stride_v=stride_v)
        dev = torch.device("cuda", rank)
        c.update_and_fetch(torch.from_numpy(K[:, :, lo:hi]).to(dev), torch.from_numpy(V[:, :, lo:hi]).to(dev))
        out = sequence_parallel_attention(torch.from_numpy(q).to(dev), c, 1 / math.sqrt(q.shape[-1]))
        torch.cuda.synchronize()
        queue.put((rank, out.float().cpu().numpy(), None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        queue.put((rank, None, repr(e)))


def tp_decoder_worker(rank, world, port, steps, queue):
    """Kv-head tensor-parallel decoder on `world` GPUs against the same decoder
    on one GPU (rank 0), same weights, context and input ids every step."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from chronoquant_mlx_b200.decoder import DecoderConfig, Qwen3StyleDecoder
        cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
        tp = Qwen3StyleDecoder(cfg, 2, 320, device=dev, seed=9, tp_group=dist.group.WORLD)
        tp.fill_context(300)
        tp.capture()
        one = None
        if rank == 0:
            one = Qwen3StyleDecoder(cfg, 2, 320, device=dev, seed=9)
            one.fill_context(300)
            one.capture()
        rels = []
        for s in range(steps):
            ids = torch.tensor([3 + s, 50 + s], device=dev)
            tp.ids.copy_(ids)
            lt = tp.decode(1).float().clone()
            if one is not None:
                one.ids.copy_(ids)
                lo = one.decode(1).float()
                rels.append(float((lt - lo).norm() / lo.norm()))
        torch.cuda.synchronize()
        del tp.graph  # graphs holding NCCL work go before the process group
        tp.close()
        if one is not None:
            del one.graph
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, rels, None))
    except Exception as e:
        queue.put((rank, None, repr(e)))


def seq_decoder_worker(rank, world, port, steps, queue):
    """Sequence-split decoder on `world` GPUs (each rank a token range of the
    context, partials merged by log-sum-exp) against the same decoder on one
    GPU (rank 0): same weights, context and input ids every step."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from chronoquant_mlx_b200.decoder import DecoderConfig, Qwen3StyleDecoder
        cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
        kw = dict(stride_k=64, stride_v=32, delta_bits_v=3, dead_zone_v=0.05)
        sp = Qwen3StyleDecoder(cfg, 1, 1100, kw, device=dev, seed=9, seq_group=dist.group.WORLD)
        sp.fill_context(1000)
        sp.capture()
        one = None
        if rank == 0:
            one = Qwen3StyleDecoder(cfg, 1, 1100, kw, device=dev, seed=9)
            one.fill_context(1000)
            one.capture()
        rels, lens = [], []
        for s in range(steps):
            ids = torch.tensor([3 + 7 * s], device=dev)
            sp.ids.copy_(ids)
            ls = sp.decode(1).float().clone()
            if one is not None:
                one.ids.copy_(ids)
                lo = one.decode(1).float()
                rels.append(float((ls - lo).norm() / lo.norm()))
        torch.cuda.synchronize()
        lens = [int(L["len"][0]) for L in sp.layers]
        del sp.graph  # graphs holding NCCL work go before the process group
        sp.close()
        if one is not None:
            del one.graph
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, rels, lens, None))
    except Exception as e:
        queue.put((rank, None, None, repr(e)))


def mesh_decoder_worker(rank, world, port, n_seq, steps, queue):
    """The decoder on a seq x tp mesh of `world` GPUs (``mesh_groups``: n_seq
    token ranges, each over world / n_seq tensor-parallel ranks) against the
    same decoder on one GPU (rank 0): same weights, context and input ids
    every step."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from chronoquant_mlx_b200.decoder import DecoderConfig, Qwen3StyleDecoder, mesh_groups
        tp_group, seq_group = mesh_groups(n_seq, world // n_seq)
        cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)
        kw = dict(stride_k=64, stride_v=32, delta_bits_v=3, dead_zone_v=0.05)
        m = Qwen3StyleDecoder(cfg, 1, 1100, kw, device=dev, seed=9, tp_group=tp_group, seq_group=seq_group)
        m.fill_context(1000)
        m.capture()
        one = None
        if rank == 0:
            one = Qwen3StyleDecoder(cfg, 1, 1100, kw, device=dev, seed=9)
            one.fill_context(1000)
            one.capture()
        rels = []
        for s in range(steps):
            ids = torch.tensor([3 + 7 * s], device=dev)
            m.ids.copy_(ids)
            lm = m.decode(1).float().clone()
            if one is not None:
                one.ids.copy_(ids)
                lo = one.decode(1).float()
                rels.append(float((lm - lo).norm() / lo.norm()))
        torch.cuda.synchronize()
        lens = [int(L["len"][0]) for L in m.layers]
        del m.graph  # graphs holding NCCL work go before the process group
        m.close()
        if one is not None:
            del one.graph
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, rels, lens, None))
    except Exception as e:
        queue.put((rank, None, None, repr(e)))


def mesh_groups_worker(rank, world, port, n_seq, queue):
    """The ranks of this rank's tensor-parallel and sequence groups on a
    n_seq x (world / n_seq) mesh (gloo, CPU)."""
    try:
        _init(rank, world, port, 60)
        from chronoquant_mlx_b200.decoder import mesh_groups
        tp_group, seq_group = mesh_groups(n_seq, world // n_seq)
        tp_ranks = dist.get_process_group_ranks(tp_group) if tp_group is not None else None
        seq_ranks = dist.get_process_group_ranks(seq_group) if seq_group is not None else None
        if seq_group is not None:  # the group carries a collective among exactly those ranks
            t = torch.tensor([rank], dtype=torch.int64)
            dist.all_reduce(t, group=seq_group)
            seq_sum = int(t.item())
        else:
            seq_sum = None
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, tp_ranks, seq_ranks, seq_sum, None))
    except Exception as e:
        queue.put((rank, None, None, None, repr(e)))


def peer_sum_worker(rank, world, port, rows, dim, queue):
    """PeerSumNorm on `world` GPUs against a torch restatement: every rank's
    part all-gathered (NCCL), summed in fp32 in rank order and rounded, added
    to x (one rounding); y = RMSNorm(x) * w as the torch expression.  Eager
    calls alternating parity, then four calls captured in a CUDA graph and
    replayed with new parts.  Returns (max ulps of x, max ulps of y)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from chronoquant_mlx_b200.peer import PeerSumNorm
        from chronoquant_mlx_b200.decoder import _rmsnorm
        ps = PeerSumNorm(dist.group.WORLD, rows, dim, device=dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        w = (1.0 + 0.1 * torch.randn(dim, generator=g, device=dev)).to(torch.bfloat16)
        dist.broadcast(w, 0)
        eps = 1e-6

        def expected(x, part):
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            acc = torch.zeros_like(part, dtype=torch.float32)
            for p in parts:
                acc += p.float()
            xe = (x.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
            return xe, _rmsnorm(xe, w, eps)

        def ulps(a, b):
            return int((a.view(torch.int16).int() - b.view(torch.int16).int()).abs().max())

        def rand_part(k):
            return (torch.randn((rows, dim), generator=g, device=dev) * (k + 1)).to(torch.bfloat16)

        worst = [0, 0]
        x = torch.randn((rows, dim), generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        for k in range(6):  # eager calls, alternating parity
            part = rand_part(k)
            xe, ye = expected(x, part)
            ps(part, x, w, eps, y, k & 1)
            torch.cuda.synchronize()
            worst[0] = max(worst[0], ulps(x, xe))
            worst[1] = max(worst[1], ulps(y, ye))
        # four calls in a graph: each replay sums the parts written before it
        parts = [rand_part(k) for k in range(4)]
        xs = [x.clone() for _ in range(4)]
        ys = [torch.empty_like(x) for _ in range(4)]
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for k in range(4):
                ps(parts[k], xs[k], w, eps, ys[k], k & 1)
        for rep in range(3):
            dist.barrier()
            x0 = [t.clone() for t in xs]
            for k in range(4):
                parts[k].copy_(rand_part(k))
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            for k in range(4):
                xe, ye = expected(x0[k], parts[k])
                worst[0] = max(worst[0], ulps(xs[k], xe))
                worst[1] = max(worst[1], ulps(ys[k], ye))
        c = ctypes.c_int(0)
        from chronoquant_mlx_b200 import _lib
        _lib.lib().cq_device_error(ctypes.byref(c), 1)
        del graph
        ps.close()
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, worst, c.value, None))
    except Exception as e:
        queue.put((rank, None, None, repr(e)))


def peer_timeout_worker(rank, world, port, queue):
    """Rank 1 never makes the call: rank 0's wait gives up (bounded) and
    cq_device_error reports 9; rank 1 stays up (its region mapped) until
    rank 0 has read the status."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        from chronoquant_mlx_b200 import _lib
        from chronoquant_mlx_b200.peer import PeerSumNorm
        ps = PeerSumNorm(dist.group.WORLD, 2, 256, device=dev)
        code = None
        if rank == 0:
            x = torch.zeros((2, 256), dtype=torch.bfloat16, device=dev)
            w = torch.ones(256, dtype=torch.bfloat16, device=dev)
            y = torch.full_like(x, 7.0)
            ps(torch.ones_like(x), x, w, 1e-6, y, 0)
            c = ctypes.c_int(0)
            _lib.lib().cq_device_error(ctypes.byref(c), 1)  # synchronises: the kernel has given up
            code = (c.value, bool(torch.all(y == 7.0)))
        dist.barrier()  # rank 1 keeps its region mapped until rank 0's kernel has given up
        dist.destroy_process_group()
        queue.put((rank, code, None))
    except Exception as e:
        queue.put((rank, None, repr(e)))


class _ShardStub:
    """The part of a cache the tail check reads: its token count."""

    def __init__(self, n):
        self.offset = n


def short_tail_worker(rank, world, port, T, q_len, stride_k, stride_v, queue):
    """sequence_parallel_attention on a sequence whose tail shard is shorter
    than the query chunk: every rank must raise ValueError before any partial
    is computed or exchanged."""
    from chronoquant_mlx_b200.distributed import sequence_parallel_attention, shard_bounds
    try:
        _init(rank, world, port, 30)
        lo, hi = shard_bounds(T, world, stride_k, stride_v)[rank]
        q = torch.zeros((1, 4, q_len, 128), dtype=torch.float16)
        try:
            sequence_parallel_attention(q, _ShardStub(hi - lo), 0.1)
            queue.put((rank, "no error", hi - lo))
        except ValueError as e:
            queue.put((rank, "raised: " + str(e), hi - lo))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the test
        queue.put((rank, "error: " + repr(e), None))
