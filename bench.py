"""Benchmark: ChronoQuant compressed-cache decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl ours|reference]

Workload (bench config 3 by default, the metric's 32k-context case): one
attention layer, B=16 sequences, 32 query / 8 KV heads, head_dim 128, a
compressed context of T=32768 tokens per sequence in the Full-Throttle V3
preset (stride_k 64, stride_v 32, INT4 K / 3-bit V residuals in INT4 lanes,
dead zones 0 / 0.05).  ``--config 2`` selects B=8, T=16384, Standard
(stride_k 32, stride_v 8, INT4, dead zone 0).  One step = append one new
token per sequence (the streaming encode) + decode attention of a bf16 query
against everything cached (the split-KV decode kernel, which also merges its
splits), issued as one replay of a CUDA graph (``DecodeGraph``) after one
copy of the step's K/V/q from a device-resident pool into the graph's flat
input buffer.  Synthetic AR(1) K/V (fp16), seeded.

value: compressed bytes the step must move (the cache's active bytes, the
reference accounting, plus query/output and the encode's own bytes) divided
by the device time per step (CUDA events, max over ranks).  The cache (~170 MB
per GPU) exceeds the 126 MB L2, so no flush is needed between steps.
e2e: the same metric through the public API with pinned host buffers: the new
token's K/V and the query copied host->device and the output device->host
inside every timed step (double-buffered: step k+1's inputs are copied in on a
copy stream while step k runs, step k's output is copied out while step k+1
runs).
roofline: the decode kernel alone, a graph of the attention launch replayed
back to back (it only reads the cache), CUDA events around the batch.

--gpus N (under torchrun, N dividing the 8 KV heads): weak scaling by KV-head
shards.  The job decodes N x B sequences; rank r holds KV heads
[r*8/N, (r+1)*8/N) (and their query heads) of every sequence, so each rank
holds as many (sequence, kv-head) units and compressed bytes as one GPU at
N=1 (591 MB for config 3, above the 126 MB L2).  No collective on the data
path: heads are independent.
--impl reference: the reference's CPU path (restated in oracle/, the
reference itself needs MLX/Metal) timed on the host cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "fused dequant-SDPA decode GB/s vs 8 TB/s HBM; decode tokens/s at 32k ctx"

CONFIGS = {
    1: dict(name="cfg1-standard-codec", B=1, Hq=32, Hkv=8, D=128, T=4096, stride_k=32, stride_v=8,
            bits_k=4, bits_v=4, dz_k=0.0, dz_v=0.0, rho_k=0.95, rho_v=0.8),
    2: dict(name="cfg2-standard-decode", B=8, Hq=32, Hkv=8, D=128, T=16384, stride_k=32, stride_v=8,
            bits_k=4, bits_v=4, dz_k=0.0, dz_v=0.0, rho_k=0.95, rho_v=0.8),
    3: dict(name="cfg3-ftv3-decode", B=16, Hq=32, Hkv=8, D=128, T=32768, stride_k=64, stride_v=32,
            bits_k=4, bits_v=3, dz_k=0.0, dz_v=0.05, rho_k=0.97, rho_v=0.85),
    4: dict(name="cfg4-standard-prefill", B=1, Hq=32, Hkv=8, D=128, T=65536, chunk=2048, stride_k=32,
            stride_v=8, bits_k=4, bits_v=4, dz_k=0.0, dz_v=0.0, rho_k=0.95, rho_v=0.8),
}
PREFILL_METRIC = "chunked prefill attention TFLOP/s over the compressed cache (config 4)"
CONFIGS[5] = dict(name="cfg5-qwen3-8b-shape-ftv3-decode", B=32, T=32768, stride_k=64, stride_v=32, bits_k=4,
                  bits_v=3, dz_k=0.0, dz_v=0.05)
DECODER_METRIC = "decode tokens/s at 32k ctx (config 5: Qwen3-8B-shape random-init decoder, FT-V3 caches)"


def active_bytes(B, H, T, D, sk, sv):
    """cache.py:274-287 active bytes for K and V at T tokens."""
    W = (D + 7) // 8
    tot = 0
    for s in (sk, sv):
        nkf = (T - 1) // s + 1 if T > 0 else 0
        npf = T - nkf
        tot += B * H * (nkf * D * 2 + npf * W * 4 + npf * 2)
    return tot


def step_bytes(cfg, T):
    """Algorithmic bytes of one decode step at T cached tokens (after append):
    attention reads the active cache + q, writes out; the encode reads the new
    K/V token and its anchor, writes codes+scale (or the anchor)."""
    B, H, Hq, D = cfg["B"], cfg["Hkv"], cfg["Hq"], cfg["D"]
    attn = active_bytes(B, H, T, D, cfg["stride_k"], cfg["stride_v"]) + 2 * B * Hq * D * 2
    t = T - 1
    enc = 0
    for s in (cfg["stride_k"], cfg["stride_v"]):
        if t % s == 0:
            enc += B * H * (D * 2 + D * 2)
        else:
            enc += B * H * (D * 2 + D * 2 + (D // 8) * 4 + 2)
    return attn, enc


def codec_bytes(cfg, B=None, H=None):
    """Algorithmic bytes of the config-1 workload (encode the whole cache, then
    one decode query): the encode reads the fp16 K and V tokens and writes the
    compressed cache (its active bytes, cache.py:274-287); the decode reads
    the compressed cache and the query and writes the output."""
    B = cfg["B"] if B is None else B
    H = cfg["Hkv"] if H is None else H
    hq = H * (cfg["Hq"] // cfg["Hkv"])
    T, D = cfg["T"], cfg["D"]
    comp = active_bytes(B, H, T, D, cfg["stride_k"], cfg["stride_v"])
    return 2 * B * H * T * D * 2 + comp + comp + 2 * B * hq * D * 2


def prefill_flops(cfg, rows=None, kv_heads=None):
    """Algorithmic FLOPs of one query chunk: 4*Hq*Tq*Tctx*D for the cached
    context plus 4*Hq*Tq^2*D/2 for the causal chunk itself (QK^T and PV, 2
    FLOPs per multiply-add).  ``rows``/``kv_heads`` restrict it to a sample."""
    Tq, Tc, D = cfg["chunk"], cfg["T"], cfg["D"]
    hq = cfg["Hq"] if kv_heads is None else kv_heads * (cfg["Hq"] // cfg["Hkv"])
    if rows is None:
        return 4 * hq * Tq * Tc * D + 4 * hq * Tq * Tq * D / 2
    # rows = the last `rows` tokens of the chunk: each sees the context plus its causal prefix
    return sum(4 * hq * (Tc + Tq - rows + i + 1) * D for i in range(rows))


def ar1_host(B, H, T, D, rho_k, rho_v, seed):
    """Seeded AR(1) K (innovation 0.31, lognormal(0,0.5) channel scale, 4
    outlier channels x8) and unit-variance AR(1) V, fp16 [B, H, T, D]."""
    g = np.random.default_rng(seed)
    chan = g.lognormal(0.0, 0.5, size=(B, H, D)).astype(np.float32)
    for b in range(B):
        for h in range(H):
            chan[b, h, g.choice(D, 4, replace=False)] *= 8.0
    K = np.empty((B, H, T, D), np.float16)
    V = np.empty((B, H, T, D), np.float16)
    k = (g.standard_normal((B, H, D)) * 0.31 / math.sqrt(1 - rho_k ** 2)).astype(np.float32)
    v = g.standard_normal((B, H, D)).astype(np.float32)
    sdv = math.sqrt(1 - rho_v ** 2)
    for t0 in range(0, T, 512):
        n = min(512, T - t0)
        ek = (g.standard_normal((n, B, H, D)) * 0.31).astype(np.float32)
        ev = (g.standard_normal((n, B, H, D)) * sdv).astype(np.float32)
        for i in range(n):
            if t0 + i:
                k = rho_k * k + ek[i]
                v = rho_v * v + ev[i]
            K[:, :, t0 + i] = k * chan
            V[:, :, t0 + i] = v
    return K, V


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report without clocks
            self.err = str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def load_peak():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(cfg_name):
    """dram bytes per decode launch from the committed ncu summary, scaled to
    this workload's active bytes (traffic grows with the cache)."""
    p = os.path.join(HERE, "profiles", "decode_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        e = d[cfg_name]
        return e
    except Exception:
        return None


# ----------------------------------------------------------------------------- GPU arm


def shard_of(cfg, world, rank):
    """KV-head shard of rank `rank` among `world` ranks (weak scaling): the
    job decodes world x B sequences and each rank holds Hkv/world KV heads of
    all of them, so every rank has the units and bytes of the one-GPU
    workload.  Returns (local batch, local kv heads, local q heads, first
    kv head)."""
    B, H, Hq = cfg["B"], cfg["Hkv"], cfg["Hq"]
    if world <= 1:
        return B, H, Hq, 0
    if H % world:
        raise SystemExit(f"--gpus {world} must divide the {H} KV heads")
    return B * world, H // world, Hq // world, rank * (H // world)


def decode_config(cfg, world, T_start):
    """The `config` object of a decode line (the same for both arms)."""
    B, H, Hq, D = cfg["B"], cfg["Hkv"], cfg["Hq"], cfg["D"]
    Bl, Hl, _, _ = shard_of(cfg, world, 0)
    return {"workload": cfg["name"], "batch": B * max(world, 1), "q_heads": Hq, "kv_heads": H, "head_dim": D,
            "context_tokens_start": T_start, "stride_k": cfg["stride_k"], "stride_v": cfg["stride_v"],
            "bits_k": cfg["bits_k"], "bits_v": cfg["bits_v"], "dead_zone_k": cfg["dz_k"], "dead_zone_v": cfg["dz_v"],
            "step": "append 1 token per (sequence, kv-head) (encode) + decode attention of one query per head",
            "l2": "cache active bytes %.0f MB per GPU > 126 MB L2; no flush" %
                  (active_bytes(Bl, Hl, T_start, D, cfg["stride_k"], cfg["stride_v"]) / 1e6),
            "parallelism": (f"one shard: all {B} sequences x {H} kv-heads" if world <= 1 else
                            f"kv-head shards over {world} GPUs: each rank holds {Hl} of {H} kv-heads of all "
                            f"{Bl} sequences (weak scaling; no collective)")}


def unit_parity(cache, cfg, unit_kv):
    """Unit (0, 0) of the benchmarked cache after all its steps, against the
    oracle (the test checker) encoding the same fp16 tokens: its state
    (anchors, packed codes, scales) bit for bit, and the halfway quotients
    (rounded half to even, codec.py:50-51) counted and the device's codes
    checked at each of them."""
    import torch
    sys.path.insert(0, HERE)
    from oracle import cq_oracle as O
    T = cache.offset
    K, V = unit_kv
    o = O.OracleCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                      delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
    sites = {}
    o.update_and_fetch(K[:, :, :T], V[:, :, :T], tie_sites=sites)
    dev = []
    for a in cache.state:
        a = a[0:1, 0:1].cpu()
        dev.append(a.view(torch.int32).numpy().view(np.uint32) if a.dtype == torch.uint32 else a.numpy())
    exact = len(dev) == len(o.state) and all(
        np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(r).view(np.uint8))
        for a, r in zip(dev, o.state))
    ties, matched = {}, True
    for comp, idx in (("k", 2), ("v", 4)):
        mask = np.concatenate(sites[comp], axis=2)
        dc = O.unpack_int4(np.ascontiguousarray(dev[idx]), cfg["D"])
        oc = O.unpack_int4(np.ascontiguousarray(o.state[idx]), cfg["D"])
        ties[comp] = int(mask.sum())
        matched = matched and bool(np.array_equal(dc[mask], oc[mask]))
    return {"unit": [0, 0], "tokens": T, "state_bit_exact_vs_oracle": bool(exact),
            "halfway_quotients": ties, "halfway_codes_match": matched}


def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    sys.path.insert(0, HERE)
    from chronoquant_mlx_b200 import ChronoQuantCache, DecodeGraph

    B, H, Hq, h0 = shard_of(cfg, world, rank)
    D, T0 = cfg["D"], cfg["T"]
    lcfg = dict(cfg, B=B, Hkv=H, Hq=Hq)  # this rank's shard
    n_new = args.warmup + args.steps + 2  # tokens appended by warm-up, timed and e2e steps
    K, V = ar1_host(B, H, T0 + 2 * n_new, D, cfg["rho_k"], cfg["rho_v"], seed=1000 + rank)
    cache = ChronoQuantCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                             delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"],
                             max_tokens=T0 + 2 * n_new + 8, page_tokens=args.page_tokens)
    # prefill (untimed) in chunks
    for t in range(0, T0, 4096):
        n = min(4096, T0 - t)
        cache.update_and_fetch(torch.from_numpy(K[:, :, t:t + n]).to(device),
                               torch.from_numpy(V[:, :, t:t + n]).to(device))
    newK = torch.from_numpy(np.ascontiguousarray(K[:, :, T0:])).to(device)
    newV = torch.from_numpy(np.ascontiguousarray(V[:, :, T0:])).to(device)
    unit_kv = (K[0:1, 0:1].copy(), V[0:1, 0:1].copy())  # the host copy of unit (0, 0), for the parity check
    del K, V
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    qs = (torch.randn((2 * n_new, B, Hq, 1, D), generator=g) / math.sqrt(D)).to(torch.bfloat16).to(device)
    scale = 1.0 / math.sqrt(D)
    # one decode step = one CUDA-graph replay: encode the new token, attend over the cache;
    # two buffer sets so the e2e loop can copy step k+1's inputs while step k runs
    dg = DecodeGraph(cache, Hq, scale, q_dtype=torch.bfloat16, max_len=T0 + 2 * n_new + 4, buffers=2)
    torch.cuda.synchronize()

    # every step's K/V/q packed in the layout of the graph's flat input buffer:
    # a step is one device-to-device copy of its inputs plus one replay
    n_in = dg.inputs.numel()
    pool = torch.empty((2 * n_new, n_in), dtype=torch.uint8, device=device)
    for j in range(2 * n_new):
        dg.keys.copy_(newK[:, :, j:j + 1])
        dg.values.copy_(newV[:, :, j:j + 1])
        dg.queries.copy_(qs[j])
        pool[j].copy_(dg.inputs)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    i_tok = [0]

    def step():
        j = i_tok[0]
        dg.inputs.copy_(pool[j], non_blocking=True)
        dg.replay()
        i_tok[0] += 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    T_start = cache.offset
    with ClockSampler(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for k in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
        dist.barrier()
    T_end = cache.offset
    tot_bytes = 0
    for T in range(T_start + 1, T_end + 1):
        a, e = step_bytes(lcfg, T)
        tot_bytes += a + e
    ms_per_step = elapsed_ms / args.steps
    value = world * tot_bytes / (elapsed_ms * 1e-3) / 1e9

    # the decode kernel alone: a graph of the attention launch only (reads the
    # cache, leaves it unchanged), replayed back to back
    attn_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(attn_graph):
        dg._attend()
    torch.cuda.synchronize()
    reps = max(100, args.steps)
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    attn_graph.replay()
    torch.cuda.synchronize()
    a0.record(stream)
    for _ in range(reps):
        attn_graph.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    mean_attn_ms = a0.elapsed_time(a1) / reps
    mean_attn_bytes = step_bytes(lcfg, cache.offset)[0]
    del attn_graph

    # e2e: the same step through the public API with host buffers -- every
    # step's K/V/q copied in from pinned host memory and its output copied
    # back to pinned host memory.  Double-buffered on a copy stream: step
    # k+1's inputs go in while step k runs, step k's output comes out while
    # step k+1 runs; the timed region ends after the last output is home.
    # each row: one step's K, V and q bytes, continuing the token sequence where the timed steps stopped
    hin = pool[i_tok[0]:].cpu().pin_memory()
    hout = torch.empty((B, Hq, 1, D), dtype=torch.bfloat16).pin_memory()
    e_steps = min(args.steps, hin.shape[0])
    copy = torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event(), torch.cuda.Event()]
    ev_done = [torch.cuda.Event(), torch.cuda.Event()]
    ev_out = [torch.cuda.Event(), torch.cuda.Event()]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    Te0 = cache.offset
    first_set = dg._cur  # buffer set of step 0
    e0.record(stream)
    copy.wait_event(e0)

    def h2d(k):  # step k's inputs into its buffer set, once step k-2 (same set) has run
        s = (first_set + k) % 2
        with torch.cuda.stream(copy):
            if k >= 2:
                copy.wait_event(ev_done[s])
            dg.inputs_of(s).copy_(hin[k], non_blocking=True)
            ev_in[s].record(copy)

    h2d(0)
    for k in range(e_steps):
        s = (first_set + k) % 2
        if k + 1 < e_steps:
            h2d(k + 1)
        stream.wait_event(ev_in[s])
        if k >= 2:
            stream.wait_event(ev_out[s])  # step k-2's output (same set) is home
        out = dg.replay()
        ev_done[s].record(stream)
        with torch.cuda.stream(copy):
            copy.wait_event(ev_done[s])
            hout.copy_(out, non_blocking=True)
            ev_out[s].record(copy)
    stream.wait_stream(copy)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    e_bytes = sum(sum(step_bytes(lcfg, T)) for T in range(Te0 + 1, cache.offset + 1))
    e2e_value = world * e_bytes / (e_ms * 1e-3) / 1e9
    h2d_bytes = hin[0].numel()
    d2h_bytes = hout.numel() * 2

    fp16_base = fp16_decode_baseline(cfg, cache.offset, device, reps) if world == 1 else None

    parity = unit_parity(cache, cfg, unit_kv) if rank == 0 else None

    peak, peak_kind = load_peak()
    achieved = mean_attn_bytes / (mean_attn_ms * 1e-3) / 1e9
    traffic = None
    tr = load_traffic(cfg["name"])
    if tr:
        traffic = tr["dram_bytes_per_launch"] * (mean_attn_bytes / tr["algorithmic_bytes_per_launch"])

    if rank == 0:
        res = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int4-residual/f16-anchor, bf16 q, f32 accumulate",
            "data": "synthetic AR(1) K/V (seeded), random bf16 queries",
            "config": decode_config(cfg, world, T_start),
            "cache_layout": {"page_tokens": cache.page_tokens, "chunk_tokens": cache.store.chunk},
            # every rank holds a head slice of all B local sequences: B tokens per step for the job
            "tokens_per_s": round(B * args.steps / (elapsed_ms * 1e-3), 1),
            "bytes_per_step_per_gpu": round(tot_bytes / args.steps),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": d2h_bytes, "steps": e_steps,
                    "copies": "pinned host <-> device on a copy stream, double-buffered (overlapping the steps)"},
            "roofline": {"bound": "hbm", "kernel": "decode_kernel (split-KV decode with in-kernel merge)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": None if traffic is None else round(traffic),
                         "algorithmic_bytes_per_launch": round(mean_attn_bytes),
                         "launch_ms": round(mean_attn_ms, 5), "launch_timing": "graph replays back to back"},
            "clocks": clk.summary(),
            "parity": parity,
            "gpu_launches": args.steps,  # one fused encode+decode kernel per graph replay
            "fp16_baseline": None if fp16_base is None else dict(
                fp16_base, compressed_bytes_per_token_kv_head=round(
                    active_bytes(1, 1, cache.offset, D, cfg["stride_k"], cfg["stride_v"]) / cache.offset, 2),
                speedup_of_compressed_kernel=round(fp16_base["ms_per_step"] / mean_attn_ms, 3)),
        }
        if not args.no_cpu_baseline and world == 1:
            res["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
        print(json.dumps(res))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_vpack3(args, cfg):
    """The decode step over a cache with physical 3-bit V codes
    (ChronoQuantCache(v_pack=3), opt-in; config 3's V codes are 3-bit),
    stepped eagerly (update_and_fetch of one token + chronoquant_sdpa, which
    runs the sm_100a decode kernel's bit-plane path), beside the same eager
    steps over the INT4-lane store.  GB/s counts the bytes each store holds
    (``physical_nbytes``: the reference's accounting cannot express 3-bit
    rows).  One GPU."""
    import torch
    sys.path.insert(0, HERE)
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa
    device = torch.device("cuda", 0)
    B, H, Hq, D, T0 = cfg["B"], cfg["Hkv"], cfg["Hq"], cfg["D"], cfg["T"]
    n = args.warmup + args.steps
    K, V = ar1_host(B, H, T0 + n, D, cfg["rho_k"], cfg["rho_v"], seed=1000)
    caches = {}
    for pack in (4, 3):
        c = ChronoQuantCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                             delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"],
                             max_tokens=T0 + n + 8, v_pack=pack)
        for t in range(0, T0, 4096):
            c.update_and_fetch(torch.from_numpy(K[:, :, t:t + min(4096, T0 - t)]).to(device),
                               torch.from_numpy(V[:, :, t:t + min(4096, T0 - t)]).to(device))
        caches[pack] = c
    newK = torch.from_numpy(np.ascontiguousarray(K[:, :, T0:])).to(device)
    newV = torch.from_numpy(np.ascontiguousarray(V[:, :, T0:])).to(device)
    del K, V
    g = torch.Generator(device="cpu").manual_seed(7)
    qs = (torch.randn((n, B, Hq, 1, D), generator=g) / math.sqrt(D)).to(torch.bfloat16).to(device)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream()
    res = {}
    for pack in (3, 4):
        c = caches[pack]
        for j in range(args.warmup):
            c.update_and_fetch(newK[:, :, j:j + 1], newV[:, :, j:j + 1])
            chronoquant_sdpa(qs[j], None, None, c, scale)
        torch.cuda.synchronize()
        T_start = c.offset
        b0 = c.physical_nbytes
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for j in range(args.warmup, n):
            c.update_and_fetch(newK[:, :, j:j + 1], newV[:, :, j:j + 1])
            out = chronoquant_sdpa(qs[j], None, None, c, scale)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        byts = (b0 + c.physical_nbytes) / 2 + 2 * B * Hq * D * 2  # mean over the steps, plus q and out
        res[pack] = dict(ms=ms, gbs=byts / (ms * 1e-3) / 1e9, T_start=T_start,
                         bytes_per_token_kv_head=round(c.physical_nbytes / (B * H * c.offset), 2),
                         reference_accounting_bytes_per_token_kv_head=round(c.nbytes / (B * H * c.offset), 2))
    r3, r4 = res[3], res[4]
    out = {
        "metric": METRIC, "value": round(r3["gbs"], 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(r3["ms"], 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "3-bit residual V (bit planes), INT4 K, f16 anchors, bf16 q, f32 accumulate",
        "data": "synthetic AR(1) K/V (seeded), random bf16 queries",
        "config": dict(decode_config(cfg, 1, r3["T_start"]), v_pack=3,
                       step="append 1 token per (sequence, kv-head) + decode attention, eager "
                            "(update_and_fetch + chronoquant_sdpa): the decode kernel's bit-plane path"),
        "bytes_per_token_kv_head": r3["bytes_per_token_kv_head"],
        "reference_accounting_bytes_per_token_kv_head": r3["reference_accounting_bytes_per_token_kv_head"],
        "int4_lanes_same_path": {"ms_per_step": round(r4["ms"], 5), "value": round(r4["gbs"], 2),
                                 "bytes_per_token_kv_head": r4["bytes_per_token_kv_head"],
                                 "note": "the same eager steps over the INT4-lane store"},
        "gpu_launches": None,
    }
    print(json.dumps(out))


def run_prefill(args, cfg):
    """Config 4: one step = encode a 2048-token chunk into the compressed cache
    (context 65536 tokens) and attend its 2048 causal queries over all 67584
    tokens on the tensor-core path (cq_append + cq_attention)."""
    import ctypes

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sys.path.insert(0, HERE)
    from chronoquant_mlx_b200 import ChronoQuantCache, _lib

    B, H, Hq, D, ctx, S = cfg["B"], cfg["Hkv"], cfg["Hq"], cfg["D"], cfg["T"], cfg["chunk"]
    T = ctx + S
    K, V = ar1_host(B, H, T, D, cfg["rho_k"], cfg["rho_v"], seed=2000 + rank)
    cache = ChronoQuantCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                             delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"],
                             max_tokens=T)
    for t in range(0, T, 4096):
        n = min(4096, T - t)
        cache.update_and_fetch(torch.from_numpy(K[:, :, t:t + n]).to(device),
                               torch.from_numpy(V[:, :, t:t + n]).to(device))
    kc = torch.from_numpy(np.ascontiguousarray(K[:, :, ctx:])).to(device)
    vc = torch.from_numpy(np.ascontiguousarray(V[:, :, ctx:])).to(device)
    del K, V
    g = torch.Generator(device="cpu").manual_seed(11 + rank)
    q = (torch.randn((B, Hq, S, D), generator=g) / math.sqrt(D)).to(torch.bfloat16).to(device)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)
    L = _lib.lib()
    desc = cache.store.descriptor()
    need = ctypes.c_size_t(0)
    _lib.check(L.cq_attention_workspace(ctypes.byref(desc), T, Hq, S, 0, ctypes.byref(need)), "bench")
    ws = torch.empty((need.value + 3) // 4, dtype=torch.float32, device=device)
    ws_bytes = ws.numel() * 4
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    ks, vs, qs = kc.stride(), vc.stride(), q.stride()

    def append(kk, vv):
        _lib.check(L.cq_append(ctypes.byref(desc), kk.data_ptr(), ks[0], ks[1], ks[2], vv.data_ptr(), vs[0], vs[1],
                               vs[2], _lib.CQ_F16, ctx, S, sp), "bench append")

    def prepare(qq):
        _lib.check(L.cq_prefill_prepare(ctypes.byref(desc), T, qq.data_ptr(), _lib.CQ_BF16, Hq, S, qs[0], qs[1],
                                        qs[2], scale, ws.data_ptr(), ws_bytes, sp), "bench prepare")

    def attend(oo):
        _lib.check(L.cq_prefill_attend(ctypes.byref(desc), T, Hq, S, 1, oo.data_ptr(), _lib.CQ_BF16, None,
                                       ws.data_ptr(), ws_bytes, sp), "bench attend")

    def step(kk, vv, qq, oo):  # the public path: encode the chunk, then cq_attention (prepare + attend)
        append(kk, vv)
        _lib.check(L.cq_attention(ctypes.byref(desc), T, qq.data_ptr(), _lib.CQ_BF16, Hq, S, 1, qs[0], qs[1],
                                  qs[2], scale, oo.data_ptr(), _lib.CQ_BF16, None, ws.data_ptr(), ws_bytes, 0, sp),
                   "bench attention")

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    for _ in range(args.warmup):
        step(kc, vc, q, out)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step(kc, vc, q, out)
        t1.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    ms_per_step = elapsed_ms / args.steps
    flops = prefill_flops(cfg) * B
    value = world * flops / (ms_per_step * 1e-3) / 1e12
    # the stages apart: encode of the chunk, tile images (history + queries), tensor-core attention
    reps = max(5, min(args.steps, 20))
    append_ms = timed(lambda: append(kc, vc), reps)
    prepare_ms = timed(lambda: prepare(q), reps)
    attend_ms = timed(lambda: attend(out), reps)

    # e2e: the chunk's K/V and the queries from pinned host memory, the output back, every step.
    # Double-buffered on a copy stream: step k+1's inputs go in while step k runs, step k's
    # output comes out while step k+1 runs; the timed region ends once the last output is home
    hk, hv, hq = kc.cpu().pin_memory(), vc.cpu().pin_memory(), q.cpu().pin_memory()
    ho = torch.empty_like(hq).pin_memory()
    sets = [(torch.empty_like(kc), torch.empty_like(vc), torch.empty_like(q), torch.empty_like(out)) for _ in range(2)]
    e_steps = max(3, min(args.steps, 10))
    copy = torch.cuda.Stream(device)
    ev_in, ev_done, ev_out = ([torch.cuda.Event(), torch.cuda.Event()] for _ in range(3))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy.wait_event(e0)

    def h2d(k):  # step k's inputs into set k % 2, once step k - 2 (same set) has run
        dk, dv, dq, _ = sets[k % 2]
        with torch.cuda.stream(copy):
            if k >= 2:
                copy.wait_event(ev_done[k % 2])
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            dq.copy_(hq, non_blocking=True)
            ev_in[k % 2].record(copy)

    h2d(0)
    for k in range(e_steps):
        dk, dv, dq, do = sets[k % 2]
        if k + 1 < e_steps:
            h2d(k + 1)
        stream.wait_event(ev_in[k % 2])
        if k >= 2:
            stream.wait_event(ev_out[k % 2])  # step k-2's output (same set) is home
        step(dk, dv, dq, do)
        ev_done[k % 2].record(stream)
        with torch.cuda.stream(copy):
            copy.wait_event(ev_done[k % 2])
            ho.copy_(do, non_blocking=True)
            ev_out[k % 2].record(copy)
    stream.wait_stream(copy)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    e2e_value = world * flops * e_steps / (e_ms * 1e-3) / 1e12

    peaks = {}
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        peak, peak_kind = float(peaks["bf16_tflops"]), "measured (burst, cuBLAS bf16)"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    achieved = flops / (attend_ms * 1e-3) / 1e12
    if rank == 0:
        res = {
            "metric": PREFILL_METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4-residual/f16-anchor cache; fp16 tensor-core operands, f32 accumulate, bf16 q/out",
            "data": "synthetic AR(1) K/V (seeded), random bf16 queries",
            "config": {"workload": cfg["name"], "batch": B, "q_heads": Hq, "kv_heads": H, "head_dim": D,
                       "context_tokens": ctx, "chunk_tokens": S, "stride_k": cfg["stride_k"],
                       "stride_v": cfg["stride_v"], "causal": True,
                       "step": "encode the chunk (cq_append) + cq_attention (tile images + tcgen05 attention)",
                       "l2": "fp16 tile images %.0f MB > 126 MB L2; no flush" % (2 * B * H * T * D * 2 / 1e6),
                       "parallelism": f"dp{world} (independent chunks per rank, no collective)"},
            "stages_ms": {"append": round(append_ms, 4), "prepare": round(prepare_ms, 4),
                          "attend": round(attend_ms, 4)},
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "steps": e_steps,
                    "h2d_bytes_per_step": (kc.numel() + vc.numel() + q.numel()) * 2,
                    "d2h_bytes_per_step": out.numel() * 2,
                    "copies": "pinned host <-> device on a copy stream, double-buffered (overlapping the steps)"},
            "roofline": {"bound": "tensor", "kernel": "attn_kernel (tcgen05 flash attention)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind, "traffic": None,
                         "algorithmic_flops_per_launch": flops, "launch_ms": round(attend_ms, 4)},
            "clocks": clk.summary(),
            "gpu_launches": args.steps * 4,  # append, unpack, query tiles, attention
        }
        if not args.no_cpu_baseline and world == 1:
            res["cpu_baseline"] = cpu_baseline_prefill(cfg, rows=args.cpu_rows)
        print(json.dumps(res))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decoder(args, cfg):
    """Config 5: greedy decode with a random-init Qwen3-8B-shape decoder (36
    layers, hidden 4096, 32/8 heads, SwiGLU 12288, vocab 151936, bf16) over
    FT-V3 compressed caches holding a 32768-token context per sequence, batch
    32.  One step = one CUDA-graph replay of all 36 layers (cuBLAS GEMMs, the
    fused append+decode kernel per layer, lm_head, argmax fed back)."""
    import ctypes

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sys.path.insert(0, HERE)
    from chronoquant_mlx_b200 import _lib
    from chronoquant_mlx_b200._tensors import cq_dtype
    from chronoquant_mlx_b200.decoder import DecoderConfig, Qwen3StyleDecoder

    B, T0 = cfg["B"], cfg["T"]
    kw = dict(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
              delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
    dc = DecoderConfig()
    n_steps = args.warmup + args.steps + 4
    t_setup = time.perf_counter()
    n_tp = n_seq = 1
    if world > 1 and args.tp and args.seqsplit:
        n_tp = args.tp_size or 2
        if world % n_tp:
            raise SystemExit(f"--tp-size {n_tp} must divide the {world} ranks")
        n_seq = world // n_tp
    elif world > 1 and args.tp:
        n_tp = world
    elif world > 1 and args.seqsplit:
        n_seq = world
    tp, split = n_tp > 1, n_seq > 1
    one_model = tp or split  # every rank runs the same sequences (else: independent replicas)
    tp_group = seq_group = None
    if one_model:
        from chronoquant_mlx_b200.decoder import mesh_groups
        tp_group, seq_group = mesh_groups(n_seq, n_tp)
    dec = Qwen3StyleDecoder(dc, B, T0 + n_steps + 4, kw, device=device, seed=100 if one_model else 100 + rank,
                            tp_group=tp_group, seq_group=seq_group, peer_sum=not args.nccl_allreduce)
    dec.fill_context(T0, seed=200 if one_model else 200 + rank)
    dec.ids.copy_(torch.arange(B, device=device) * 7 + 1)
    dec.capture()
    setup_s = time.perf_counter() - t_setup
    stream = torch.cuda.current_stream()
    dec.decode(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    bytes_step = dec.bytes_per_step()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.decode(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    value = (1 if one_model else world) * B / (ms * 1e-3)

    # the attention kernels alone: a graph of every layer's read-only attention
    q = torch.zeros((B, dec.heads, dc.head_dim), device=device, dtype=torch.bfloat16)
    qs = q.stride()
    lib = _lib.lib()
    ag = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ag):
        for L in dec.layers:
            _lib.check(lib.cq_attention_at(ctypes.byref(L["desc"]), L["len"].data_ptr(), dec.max_len, q.data_ptr(),
                                           cq_dtype(q), dec.heads, qs[0], qs[1], 1.0 / math.sqrt(dc.head_dim),
                                           dec.attn_out.data_ptr(), cq_dtype(dec.attn_out), None,
                                           dec.workspace.data_ptr(), dec.workspace.numel() * 4,
                                           torch.cuda.current_stream().cuda_stream), "bench")
    ag.replay()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    a0.record(stream)
    for _ in range(reps):
        ag.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / reps
    cache_bytes = sum(L["cache"].nbytes for L in dec.layers)
    del ag

    # the collectives of a step alone, each set captured as a graph and replayed: the per-layer
    # partial exchange + merge of the sequence split, the two all-reduces per layer of the
    # tensor-parallel split (every rank runs the same captures in the same order)
    comm = {}
    if split:
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg):
            for _ in dec.layers:
                dec._merge_partials()
        cg.replay()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(reps):
            cg.replay()
        c1.record(stream)
        torch.cuda.synchronize()
        comm["seq_allgather_merge_ms_per_step"] = round(c0.elapsed_time(c1) / reps, 4)
        del cg
    if tp:
        xr = torch.zeros((B, dc.hidden), device=device, dtype=torch.bfloat16)
        yr, pr = torch.empty_like(xr), torch.zeros_like(xr)
        ln = dec.layers[0]["ln2"]
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg):
            for k in range(2 * dc.layers):
                if dec.peer is not None:  # the fused peer sum + residual + RMSNorm of the step
                    dec.peer(pr, xr, ln, dc.eps, yr, k & 1)
                else:
                    dec._reduce(xr)
        cg.replay()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(reps):
            cg.replay()
        c1.record(stream)
        torch.cuda.synchronize()
        comm["tp_peer_sum_norm_ms_per_step" if dec.peer is not None else "tp_allreduce_ms_per_step"] = round(
            c0.elapsed_time(c1) / reps, 4)
        del cg

    # e2e: a host-driven serving loop -- every step's input ids copied in from pinned host
    # memory, the sampled ids copied back and waited for, so the host holds each token before
    # it feeds the next step
    hin = torch.empty(B, dtype=torch.long).pin_memory()
    hout = torch.empty(B, dtype=torch.long).pin_memory()
    hin.copy_(dec.ids.cpu())
    e_steps = 3
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for _ in range(e_steps):
        dec.ids.copy_(hin, non_blocking=True)
        dec.decode(1)
        hout.copy_(dec.out_ids, non_blocking=True)
        stream.synchronize()
        hin.copy_(hout)
    x1.record(stream)
    torch.cuda.synchronize()
    e_ms = x0.elapsed_time(x1) / e_steps
    if world > 1:
        tt = torch.tensor([e_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    peak, peak_kind = load_peak()
    tp_sum = ("one kernel: peer-memory sum over NVLink + residual add + RMSNorm" if dec.peer is not None else
              "NCCL all-reduce")
    if rank == 0:
        res = {
            "metric": DECODER_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong" if one_model else "weak", "vs_baseline": None,
            "dtype": "bf16 weights/activations, int4-residual/f16-anchor FT-V3 caches, f32 accumulate",
            "data": "random-init weights N(0,0.02); synthetic seeded K/V context encoded by the cache; greedy ids",
            "config": {"workload": cfg["name"], "batch": B, "context_tokens": T0, "layers": dc.layers,
                       "hidden": dc.hidden, "q_heads": dc.heads, "kv_heads": dc.kv_heads, "head_dim": dc.head_dim,
                       "ffn": dc.ffn, "vocab": dc.vocab, "caches": "FT-V3 (64/32, 4/3 bits, dz 0/0.05)",
                       "step": "one CUDA-graph replay: 36 x (RMSNorm, QKV, q/k norm, RoPE, fused append+decode "
                               "attention, o_proj, SwiGLU) + lm_head + argmax",
                       "parallelism": (f"seq{n_seq} x tp{n_tp} ({n_seq} token ranges of the context, each over "
                                       f"{n_tp} kv-head tensor-parallel ranks: {tp_sum} after o_proj and the "
                                       "down projection within a range, all-gather of partial attention + "
                                       "log-sum-exp merge per layer across ranges)") if tp and split else
                                      (f"tp{world} (kv-head tensor parallel, {tp_sum} after o_proj and "
                                       "the down projection)") if tp else
                                      (f"seq{world} (token ranges of one sequence per rank, NCCL all-gather of "
                                       "partial attention + log-sum-exp merge per layer)") if split else
                                      f"dp{world} (independent replicas)",
                       "setup_seconds": round(setup_s, 1)},
            "attention_ms_per_step": round(attn_ms, 4),
            "collectives": comm or None,
            "compressed_cache_bytes": cache_bytes,
            "e2e": {"value": round((1 if one_model else world) * B / (e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": hin.numel() * hin.element_size(),
                    "d2h_bytes_per_step": hout.numel() * hout.element_size(), "steps": e_steps},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (weights + compressed caches, each read once)",
                         "achieved": round(bytes_step / (ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bytes_step / (ms * 1e-3) / 1e9 / peak, 4), "peak_source": peak_kind,
                         "traffic": None, "algorithmic_bytes_per_step": bytes_step},
            "clocks": clk.summary(),
            # this package's kernels per step: per layer two RMSNorms, q/k norm + RoPE, the fused
            # append+decode kernel (or the read-only attention) and SwiGLU, plus the partial merge
            # under a sequence split; one final RMSNorm
            "gpu_launches": args.steps * ((6 if split else 5) * dc.layers + 1),
        }
        print(json.dumps(res))
    if world > 1:
        dec.graph = None  # graphs holding NCCL work go before the process group
        torch.cuda.synchronize()
        dec.close()
        dist.barrier()
        dist.destroy_process_group()


def _prefill_unit(cfg, seed, rows):
    """One kv-head of config 4 on the reference's CPU path (oracle port):
    encode the chunk onto the cached context (cache.py:87-129), reconstruct
    the fp16 history (cache.py:131-160), fallback SDPA (attention.py:61-74)
    for the last ``rows`` queries of the chunk.  Returns (seconds, flops)."""
    from oracle import cq_oracle as O
    ctx, S, D = cfg["T"], cfg["chunk"], cfg["D"]
    rep = cfg["Hq"] // cfg["Hkv"]
    K, V = ar1_host(1, 1, ctx + S, D, cfg["rho_k"], cfg["rho_v"], seed)
    c = O.OracleCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                      delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
    c.update_and_fetch(K[:, :, :ctx], V[:, :, :ctx])
    q = (np.random.default_rng(seed).standard_normal((1, rep, rows, D)) / math.sqrt(D)).astype(np.float32)
    q = O.round_bf16(q)
    t0 = time.perf_counter()
    c.update_and_fetch(K[:, :, ctx:], V[:, :, ctx:])
    fk, fv = c.reconstruct_history()
    mask = O.causal_mask(S, ctx + S)[S - rows:]
    O.fallback_sdpa(q, "bf16", fk, fv, 1.0 / math.sqrt(D), mask)
    return time.perf_counter() - t0, prefill_flops(cfg, rows=rows, kv_heads=1)


def _prefill_worker(a):
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):  # one BLAS thread per process: the processes are the parallelism
        return _prefill_unit(*a)


def cpu_baseline_prefill(cfg, rows=128):
    sys.path.insert(0, HERE)
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):
        sec, fl = _prefill_unit(cfg, 0, rows)
    return {"value": round(fl / sec / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"1 of {cfg['Hkv']} kv-heads, the last {rows} of {cfg['chunk']} queries: oracle chunk encode "
                      f"+ fp16 reconstruct of {cfg['T'] + cfg['chunk']} tokens + fallback SDPA (numpy)",
            "seconds": round(sec, 2), "host_cpus": os.cpu_count()}


def _count_kernels(fn):
    """Kernels one call of ``fn`` launches on the GPU (torch profiler, outside
    any timed region; copies and memsets are not kernels)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
    return [n for n in names if not n.lower().startswith(("memcpy", "memset"))]


def run_codec(args, cfg):
    """Config 1 on the GPU: encode the whole cache (B1, Hkv8, T4096, Standard)
    through ``update_and_fetch``, then one decode query through
    ``chronoquant_sdpa`` (the fused path of attention.py:44-59).  Both calls
    are captured once as a CUDA graph over a preallocated cache; a replay
    re-encodes every token into the same pages and decodes, so each step does
    the whole workload.  The inputs and cache (~22 MB) fit in L2, so the L2 is
    flushed (a 256 MB write) before every timed step and each step is timed
    alone with CUDA events.  e2e: K, V and the query copied in from pinned
    host memory and the output copied back inside every timed step."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sys.path.insert(0, HERE)
    from chronoquant_mlx_b200 import ChronoQuantCache, chronoquant_sdpa

    B, H, Hq, _ = shard_of(cfg, world, rank)
    D, T = cfg["D"], cfg["T"]
    K, V = ar1_host(B, H, T, D, cfg["rho_k"], cfg["rho_v"], seed=0 + rank)
    g = np.random.default_rng(rank)
    q_host = (g.standard_normal((B, Hq, 1, D)) / math.sqrt(D)).astype(np.float16)
    k_dev = torch.from_numpy(K).to(device)
    v_dev = torch.from_numpy(V).to(device)
    q_dev = torch.from_numpy(q_host).to(device)
    scale = 1.0 / math.sqrt(D)
    cache = ChronoQuantCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                             delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"],
                             max_tokens=T, page_tokens=args.page_tokens)
    out_box = [None]

    def workload():
        cache.offset = 0  # re-encode from the first token into the same pages
        kk, vv = cache.update_and_fetch(k_dev, v_dev)
        out_box[0] = chronoquant_sdpa(q_dev, kk, vv, cache, scale)

    workload()  # allocates the store and the attention workspace
    kernels = _count_kernels(workload)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        workload()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        workload()
    out = out_box[0]
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed_steps(n, inputs_in=None, output_out=None):
        """n steps, each after an L2 flush and timed alone; inputs_in /
        output_out (host copies) run inside each step's events."""
        ms = []
        for _ in range(n):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if inputs_in is not None:
                inputs_in()
            graph.replay()
            if output_out is not None:
                output_out()
            e1.record(stream)
            ms.append((e0, e1))
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in ms]

    timed_steps(args.warmup)
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        ms = timed_steps(args.steps)
    elapsed_ms = sum(ms)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    ms_per_step = elapsed_ms / args.steps
    byts = codec_bytes(cfg, B, H)
    value = world * byts / (ms_per_step * 1e-3) / 1e9

    # the encode kernel alone (the larger share of the bytes), L2 flushed before each launch
    enc_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(enc_graph):
        cache.offset = 0
        cache.update_and_fetch(k_dev, v_dev)
    cache.offset = T
    enc = []
    for _ in range(max(20, args.steps)):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        enc_graph.replay()
        e1.record(stream)
        enc.append((e0, e1))
    torch.cuda.synchronize()
    enc_ms = statistics.mean(a.elapsed_time(b) for a, b in enc)
    comp = active_bytes(B, H, T, D, cfg["stride_k"], cfg["stride_v"])
    enc_bytes = 2 * B * H * T * D * 2 + comp

    # e2e through the public API from pinned host memory
    hk = torch.from_numpy(K).pin_memory()
    hv = torch.from_numpy(V).pin_memory()
    hq = torch.from_numpy(q_host).pin_memory()
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def h2d():
        k_dev.copy_(hk, non_blocking=True)
        v_dev.copy_(hv, non_blocking=True)
        q_dev.copy_(hq, non_blocking=True)

    def d2h():
        hout.copy_(out, non_blocking=True)

    e_ms = timed_steps(args.steps, inputs_in=h2d, output_out=d2h)
    e_tot = sum(e_ms)
    if world > 1:
        tt = torch.tensor([e_tot], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_tot = float(tt.item())
    e2e_value = world * byts / (e_tot / args.steps * 1e-3) / 1e9

    # parity of this run's output and state against the oracle (the test checker)
    parity = None
    cpu = None
    if rank == 0:
        from oracle import cq_oracle as O
        o = O.OracleCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                          delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
        sites = {}
        o.update_and_fetch(K, V, tie_sites=sites)
        dev = []
        for a in cache.state:
            a = a.cpu()
            dev.append(a.view(torch.int32).numpy().view(np.uint32) if a.dtype == torch.uint32 else a.numpy())
        exact = all(np.array_equal(np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(r).view(np.uint8))
                    for a, r in zip(dev, o.state))
        # B=1, q_len=1 dispatches to the fused kernel (attention.py:44-59): q pre-scaled in fp16
        qs = (q_host.astype(np.float64) * float(np.float16(scale))).astype(np.float16).astype(np.float32)
        kk, kv, pk, sk, pv, sv = o.state
        ref = O.fused_decode(qs[0, :, 0], kk[0], pk[0], sk[0], kv[0], pv[0], sv[0], T, cfg["stride_k"],
                             cfg["stride_v"], D)[None, :, None, :]
        got = out.float().cpu().numpy()
        err = np.abs(got - ref)
        ties = {c: int(np.concatenate(sites[c], axis=2).sum()) for c in ("k", "v")}
        parity = {"state_bit_exact_vs_oracle": bool(exact), "halfway_quotients": ties,
                  "attention_max_abs_err_vs_oracle": float(err.max()),
                  "attention_within_2e-3_1e-2": bool((err <= 2e-3 + 1e-2 * np.abs(ref)).all())}
        if not args.no_cpu_baseline:
            cpu = cpu_baseline_codec(cfg, args.cpu_budget)

    peak, peak_kind = load_peak()
    achieved = enc_bytes / (enc_ms * 1e-3) / 1e9
    if rank == 0:
        res = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4-residual/f16-anchor, fp16 K/V/q, f32 accumulate",
            "data": "synthetic AR(1) K/V (seeded 0), q ~ N(0,1)/sqrt(128)",
            "config": {"workload": cfg["name"], "batch": cfg["B"] * max(world, 1), "q_heads": cfg["Hq"],
                       "kv_heads": cfg["Hkv"], "head_dim": D, "tokens": T, "stride_k": cfg["stride_k"],
                       "stride_v": cfg["stride_v"], "bits_k": cfg["bits_k"], "bits_v": cfg["bits_v"],
                       "dead_zone_k": cfg["dz_k"], "dead_zone_v": cfg["dz_v"],
                       "step": "encode all T tokens of every (sequence, kv-head) + one decode query per q head "
                               "(one CUDA-graph replay)",
                       "l2": "inputs + cache ~%.0f MB < 126 MB L2: 256 MB L2 flush before every timed step"
                             % ((2 * B * H * T * D * 2 + comp) / 1e6),
                       "parallelism": "one GPU" if world <= 1 else f"kv-head shards over {world} GPUs (weak)"},
            "bytes_per_step_per_gpu": byts,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": hk.numel() * 2 + hv.numel() * 2 + hq.numel() * 2,
                    "d2h_bytes_per_step": hout.numel() * hout.element_size(),
                    "copies": "pinned host -> device before, device -> host after each step, in the timed region"},
            "roofline": {"bound": "hbm", "kernel": "append_block_kernel (encode of all tokens)", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": None, "algorithmic_bytes_per_launch": enc_bytes, "launch_ms": round(enc_ms, 5),
                         "launch_timing": "one launch at a time, L2 flushed before each"},
            "clocks": clk.summary(),
            "parity": parity,
            "gpu_launches": len(kernels) * args.steps,
            "kernels_per_step": kernels,
            "cpu_baseline": cpu,
        }
        print(json.dumps(res))
    del graph, enc_graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _codec_unit(cfg, K, V, q, scale):
    """The config-1 workload of one (sequence, kv-head) on the reference's CPU
    path: encode all tokens (cache.py:87-129), reconstruct the fp16 history
    (cache.py:131-160), the fallback SDPA of its query heads (attention.py:61-74)."""
    from oracle import cq_oracle as O
    c = O.OracleCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                      delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
    c.update_and_fetch(K, V)
    fk, fv = c.reconstruct_history()
    return O.fallback_sdpa(q, "f16", fk, fv, scale, None)


def cpu_baseline_codec(cfg, budget_s=15.0):
    """The whole config-1 workload on the oracle, one host thread."""
    sys.path.insert(0, HERE)
    from threadpoolctl import threadpool_limits
    K, V = ar1_host(cfg["B"], cfg["Hkv"], cfg["T"], cfg["D"], cfg["rho_k"], cfg["rho_v"], seed=0)
    q = (np.random.default_rng(0).standard_normal((cfg["B"], cfg["Hq"], 1, cfg["D"])) /
         math.sqrt(cfg["D"])).astype(np.float16)
    scale = 1.0 / math.sqrt(cfg["D"])
    n, t_tot = 0, 0.0
    with threadpool_limits(1):
        _codec_unit(cfg, K, V, q, scale)
        while t_tot < budget_s and n < 30:
            t0 = time.perf_counter()
            _codec_unit(cfg, K, V, q, scale)
            t_tot += time.perf_counter() - t0
            n += 1
    return {"value": round(n * codec_bytes(cfg) / t_tot / 1e9, 5), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"the whole workload {n} times: oracle encode of {cfg['T']} tokens x {cfg['Hkv']} kv-heads + "
                      "fp16 reconstruct + fallback SDPA (numpy, 1 thread)",
            "ms_per_step": round(1e3 * t_tot / n, 2), "host_cpus": os.cpu_count()}


_CODEC_DATA = {}


def _codec_init(cfg):
    """Pool initializer: every worker generates the workload's inputs once."""
    sys.path.insert(0, HERE)
    K, V = ar1_host(cfg["B"], cfg["Hkv"], cfg["T"], cfg["D"], cfg["rho_k"], cfg["rho_v"], seed=0)
    rep = cfg["Hq"] // cfg["Hkv"]
    q = (np.random.default_rng(0).standard_normal((cfg["B"], cfg["Hq"], 1, cfg["D"])) /
         math.sqrt(cfg["D"])).astype(np.float16)
    for h in range(cfg["Hkv"]):
        _CODEC_DATA[h] = (np.ascontiguousarray(K[:, h:h + 1]), np.ascontiguousarray(V[:, h:h + 1]),
                          np.ascontiguousarray(q[:, h * rep:(h + 1) * rep]))


def _codec_worker(a):
    cfg, h = a
    K, V, q = _CODEC_DATA[h]
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):  # one BLAS thread per process: the processes are the parallelism
        t0 = time.perf_counter()
        _codec_unit(cfg, K, V, q, 1.0 / math.sqrt(cfg["D"]))
        return time.perf_counter() - t0


def run_reference_codec(args, cfg):
    """Config 1 on the reference's CPU path (oracle restatement) with the host
    cores: one process per kv-head; a step is the whole workload (every
    kv-head's encode, reconstruct and SDPA) and is timed by the wall clock."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp
    workers = max(1, min(os.cpu_count() or 1, cfg["Hkv"]))
    tasks = [(cfg, h) for h in range(cfg["Hkv"])]
    ctx = mp.get_context("spawn")
    with ctx.Pool(workers, initializer=_codec_init, initargs=(cfg,)) as pool:
        for _ in range(args.warmup):
            pool.map(_codec_worker, tasks, chunksize=1)
        ms = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            pool.map(_codec_worker, tasks, chunksize=1)
            ms.append(1e3 * (time.perf_counter() - t0))
    mean = sum(ms) / len(ms)
    value = codec_bytes(cfg) / (mean * 1e-3) / 1e9
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4-residual/f16-anchor, fp16 fallback SDPA",
        "data": "synthetic AR(1) K/V (seeded 0)",
        "config": {"workload": cfg["name"], "batch": cfg["B"], "q_heads": cfg["Hq"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "tokens": cfg["T"], "stride_k": cfg["stride_k"],
                   "stride_v": cfg["stride_v"], "bits_k": cfg["bits_k"], "bits_v": cfg["bits_v"],
                   "dead_zone_k": cfg["dz_k"], "dead_zone_v": cfg["dz_v"],
                   "parallelism": f"{workers} host processes, one kv-head each"},
        "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": workers, "kind": "port",
                         "sample": "the whole workload each step (oracle restatement of the reference's encode + "
                                   "fp16 reconstruct + fallback SDPA; MLX/Metal is unavailable here)"},
        "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def run_reference_prefill(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import multiprocessing as mp
    workers = max(1, min(os.cpu_count() or 1, cfg["Hkv"]))
    ctx = mp.get_context("spawn")
    t0 = time.perf_counter()
    with ctx.Pool(workers) as pool:
        res = pool.map(_prefill_worker, [(cfg, 300 + i, args.cpu_rows) for i in range(workers)])
    wall = time.perf_counter() - t0
    sec = max(r[0] for r in res)
    fl = sum(r[1] for r in res)
    value = fl / sec / 1e12
    out = {
        "impl": "reference", "metric": PREFILL_METRIC, "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": world, "steps": 1, "warmup": 0, "ms_per_step": round(prefill_flops(cfg) / (value * 1e12) * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 reconstruct, fp32 scores (bf16 q x fp16 K), numpy", "data": "synthetic AR(1) K/V (seeded)",
        "config": {"workload": cfg["name"], "batch": cfg["B"], "q_heads": cfg["Hq"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "context_tokens": cfg["T"], "chunk_tokens": cfg["chunk"],
                   "parallelism": f"{workers} host processes"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": workers, "kind": "port",
                         "sample": f"{workers} kv-heads x the last {args.cpu_rows} queries each (oracle restatement of "
                                   "the reference's encode + fp16 reconstruct + fallback SDPA); wall %.1f s" % wall},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def fp16_decode_baseline(cfg, T, device, reps):
    """Decode attention of the same shape over an uncompressed fp16 cache (the
    FlashDecoding baseline of bench config 3): flash_attn_with_kvcache when
    it runs on this GPU, else torch SDPA with GQA.  Times `reps` calls back to
    back with CUDA events; reports bytes per token and kv-head (K+V) and the
    fp16 cache read rate."""
    import torch
    import torch.nn.functional as F
    B, H, Hq, D = cfg["B"], cfg["Hkv"], cfg["Hq"], cfg["D"]
    g = torch.Generator(device=device).manual_seed(5)
    k = torch.randn((B, T, H, D), generator=g, device=device, dtype=torch.float16)
    v = torch.randn((B, T, H, D), generator=g, device=device, dtype=torch.float16)
    q = (torch.randn((B, 1, Hq, D), generator=g, device=device) / math.sqrt(D)).to(torch.float16)
    impl, fn = None, None
    try:
        from flash_attn import flash_attn_with_kvcache
        flash_attn_with_kvcache(q, k, v, causal=False)
        torch.cuda.synchronize()
        impl, fn = "flash_attn_with_kvcache (flash-attn 2)", lambda: flash_attn_with_kvcache(q, k, v, causal=False)
    except Exception as e:  # not built for this GPU
        torch.cuda.synchronize()
        note = f"flash_attn unavailable ({type(e).__name__})"
        kt, vt, qt = k.transpose(1, 2), v.transpose(1, 2), q.transpose(1, 2)
        impl = f"torch SDPA, enable_gqa ({note})"
        fn = lambda: F.scaled_dot_product_attention(qt, kt, vt, enable_gqa=True)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    fp16_bytes = 2 * B * H * T * D * 2
    del k, v
    return {"impl": impl, "ms_per_step": round(ms, 5), "fp16_bytes_per_token_kv_head": 2 * D * 2,
            "fp16_cache_gbs": round(fp16_bytes / (ms * 1e-3) / 1e9, 1), "tokens": T}


# ----------------------------------------------------------------------------- CPU reference arm


def _ref_unit_setup(cfg, seed):
    from oracle import cq_oracle as O
    K, V = ar1_host(1, 1, cfg["T"] + 64, cfg["D"], cfg["rho_k"], cfg["rho_v"], seed)
    c = O.OracleCache(stride_k=cfg["stride_k"], stride_v=cfg["stride_v"], delta_bits_k=cfg["bits_k"],
                      delta_bits_v=cfg["bits_v"], dead_zone_k=cfg["dz_k"], dead_zone_v=cfg["dz_v"])
    c.update_and_fetch(K[:, :, :cfg["T"]], V[:, :, :cfg["T"]])
    return c, K, V


def _ref_unit_step(c, K, V, q, scale):
    """One decode step of one (sequence, kv-head) unit on the reference's CPU
    path: encode the new token (cache.py:87-129), reconstruct the fp16 history
    (cache.py:131-160) and the fallback GQA SDPA (attention.py:61-74)."""
    from oracle import cq_oracle as O
    t = c.offset
    c.update_and_fetch(K[:, :, t:t + 1], V[:, :, t:t + 1])
    fk, fv = c.reconstruct_history()
    return O.fallback_sdpa(q, "f16", fk, fv, scale, None)


def _ref_worker(args):
    cfg, seed, n_steps = args
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):  # one BLAS thread per process: the processes are the parallelism
        return _ref_worker_steps(cfg, seed, n_steps)


def _ref_worker_steps(cfg, seed, n_steps):
    c, K, V = _ref_unit_setup(cfg, seed)
    rep = cfg["Hq"] // cfg["Hkv"]
    q = (np.random.default_rng(seed).standard_normal((1, rep, 1, cfg["D"])) / math.sqrt(cfg["D"])).astype(np.float16)
    times = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        _ref_unit_step(c, K, V, q, 1.0 / math.sqrt(cfg["D"]))
        times.append(time.perf_counter() - t0)
    return times, c.offset


def cpu_baseline(cfg, budget_s=20.0):
    """The oracle's reference-structured decode step on one (sequence,
    kv-head) unit, single thread, GB/s of that unit's compressed bytes."""
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):
        return _cpu_baseline_1t(cfg, budget_s)


def _cpu_baseline_1t(cfg, budget_s):
    sys.path.insert(0, HERE)
    c, K, V = _ref_unit_setup(cfg, 0)
    rep = cfg["Hq"] // cfg["Hkv"]
    q = (np.random.default_rng(0).standard_normal((1, rep, 1, cfg["D"])) / math.sqrt(cfg["D"])).astype(np.float16)
    scale = 1.0 / math.sqrt(cfg["D"])
    _ref_unit_step(c, K, V, q, scale)
    n, t_tot, byts = 0, 0.0, 0
    while t_tot < budget_s and n < 60:
        t0 = time.perf_counter()
        _ref_unit_step(c, K, V, q, scale)
        t_tot += time.perf_counter() - t0
        unit_cfg = dict(cfg, B=1, Hkv=1, Hq=rep)
        a, e = step_bytes(unit_cfg, c.offset)
        byts += a + e
        n += 1
    return {"value": round(byts / t_tot / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{n} decode steps of 1 of {cfg['B'] * cfg['Hkv']} (sequence, kv-head) units at "
                      f"T={cfg['T']}: oracle encode + fp16 reconstruct + fallback SDPA (numpy, 1 thread)",
            "seconds": round(t_tot, 2), "host_cpus": os.cpu_count()}


def run_reference(args, cfg):
    """The reference's CPU path (oracle restatement) on the host cores: one
    process per core, each stepping one (sequence, kv-head) unit of the
    workload.  A step of this arm is one decode step of `workers` units in
    parallel (a bounded sample of the workload's units); `ms_per_step` and
    `value` are that sample's own measured time and throughput."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    # time one unit-step to size each step's sample (whole run within ~2 minutes)
    sys.path.insert(0, HERE)
    c, K, V = _ref_unit_setup(cfg, 0)
    rep = cfg["Hq"] // cfg["Hkv"]
    q = (np.random.default_rng(0).standard_normal((1, rep, 1, cfg["D"])) / math.sqrt(cfg["D"])).astype(np.float16)
    t0 = time.perf_counter()
    _ref_unit_step(c, K, V, q, 1.0 / math.sqrt(cfg["D"]))
    t_unit = time.perf_counter() - t0
    total_steps = args.steps + args.warmup
    units = cfg["B"] * cfg["Hkv"] * max(world, 1)
    workers = min(cores, units)
    # steps per worker so that the whole timed run stays near 90 s of wall time
    per_worker_steps = max(2, min(total_steps, 60, int(90.0 / max(t_unit, 1e-3))))  # K/V hold T + 64 tokens
    ctx = mp.get_context("spawn")
    t_wall = time.perf_counter()
    with ctx.Pool(workers) as pool:
        res = pool.map(_ref_worker, [(cfg, 100 + i, per_worker_steps) for i in range(workers)])
    t_wall = time.perf_counter() - t_wall
    w = min(args.warmup, per_worker_steps - 1)
    timed = per_worker_steps - w
    # step i of the sample = every worker's i-th unit step, run in parallel: its time is the slowest worker's
    step_ms = [1e3 * max(times[w + i] for times, _ in res) for i in range(timed)]
    ms = sum(step_ms) / timed
    unit_cfg = dict(cfg, B=1, Hkv=1, Hq=rep)
    byts = sum(step_bytes(unit_cfg, cfg["T"] + w + i + 1)[0] + step_bytes(unit_cfg, cfg["T"] + w + i + 1)[1]
               for i in range(timed)) / timed
    value = workers * byts / (ms * 1e-3) / 1e9
    sample = (f"each step: one decode step (encode the new token, fp16 reconstruct, fallback SDPA) on each of "
              f"{workers} of the workload's {units} (sequence, kv-head) units, one host process per unit "
              f"(oracle restatement of the reference's CPU path; MLX/Metal is unavailable here); {timed} timed "
              f"steps after {w} warm-up, wall {t_wall:.1f} s")
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": timed, "warmup": w, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4-residual/f16-anchor, fp16 fallback SDPA", "data": "synthetic AR(1) K/V (seeded)",
        "config": decode_config(cfg, world, cfg["T"] + w),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": workers, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--page-tokens", type=int, default=None, help="cache page size (default: the cache's choice)")
    ap.add_argument("--cpu-rows", type=int, default=128, help="config 4 CPU sample: query rows per kv-head")
    ap.add_argument("--tp", action="store_true", help="config 5 under torchrun: kv-head tensor parallel")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="config 5 tensor parallel: NCCL all-reduce + separate add and RMSNorm instead of the fused "
                         "peer-memory sum")
    ap.add_argument("--tp-size", type=int, default=None,
                    help="config 5 with --tp and --seqsplit: tensor-parallel ranks per token range (the mesh is "
                         "(N / tp-size) token ranges x tp-size; default 2)")
    ap.add_argument("--seqsplit", action="store_true",
                    help="config 5: one sequence (batch 1, 524288-token context unless --context), split by "
                         "token ranges over the torchrun ranks")
    ap.add_argument("--v-pack", type=int, default=4, choices=[3, 4],
                    help="decode configs: 3 = physical 3-bit V codes (ChronoQuantCache(v_pack=3), opt-in; needs "
                         "3-bit V codes, i.e. config 3), stepped eagerly beside the INT4-lane store")
    ap.add_argument("--context", type=int, default=None,
                    help="config 4: cached tokens before the chunk (default 65536; smaller for profiler "
                         "captures); config 5: context tokens")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = CONFIGS[args.config]
    if args.config == 4 and args.context is not None:
        cfg = dict(cfg, T=args.context, name=f"{cfg['name']}-ctx{args.context}")
    if args.config == 5 and args.seqsplit:
        T = args.context or 524288
        cfg = dict(cfg, B=1, T=T, name=f"cfg5-qwen3-8b-shape-ftv3-seqsplit-{T}")
    elif args.config == 5 and args.context is not None:
        cfg = dict(cfg, T=args.context, name=f"{cfg['name']}-ctx{args.context}")
    if args.config == 5:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 5 is a 36-layer 8B decoder; the reference's "
                              "CPU path (numpy oracle) cannot run it in a bounded sample"}))
        else:
            run_decoder(args, cfg)
        return
    if args.config == 1:
        if args.impl == "reference":
            run_reference_codec(args, cfg)
        else:
            run_codec(args, cfg)
        return
    if args.config == 4:
        if args.impl == "reference":
            run_reference_prefill(args, cfg)
        else:
            run_prefill(args, cfg)
        return
    if args.v_pack == 3:
        if cfg["bits_v"] > 3:
            ap.error("--v-pack 3 needs 3-bit V codes (config 3)")
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no physical 3-bit format "
                              "(README.md:57); its arm is the INT4-lane config 3 line"}))
        else:
            run_vpack3(args, cfg)
        return
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
