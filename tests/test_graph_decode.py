"""DecodeGraph: the decode step captured once as a CUDA graph and replayed at
growing lengths equals the eager step (update_and_fetch + chronoquant_sdpa)
on an identical cache -- the cache bytes bit for bit, the attention within
max-abs 2e-3 / relative 1e-2 (different split boundaries round differently)."""

import math

import numpy as np
import pytest
import torch

from oracle import cq_oracle as O

ATOL, RTOL = 2e-3, 1e-2


def _close(a, b):
    a = a.detach().float().cpu().numpy().astype(np.float64)
    b = b.detach().float().cpu().numpy().astype(np.float64)
    err = np.abs(a - b)
    assert (err <= ATOL + RTOL * np.abs(b)).all(), f"max abs err {err.max():.3e}"


def test_decode_graph_is_exported():
    from chronoquant_mlx_b200 import DecodeGraph
    assert callable(DecodeGraph)


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hkv,Hq,T,sk,sv,steps,headroom,v_pack", [
    (2, 2, 8, 500, 32, 8, 40, 0, 4),     # crosses I-frames of both strides and a chunk boundary
    (1, 4, 16, 1000, 64, 32, 70, 0, 4),  # Full-Throttle strides, crosses a page boundary
    # a graph sized for far more tokens than are cached: the launch has more warps than the
    # current length has chunks, and only as many as there are chunks take work
    (1, 2, 8, 300, 64, 32, 12, 20000, 4),
    (2, 2, 8, 100, 32, 8, 8, 3000, 4),
    # physical 3-bit V codes: the step kernel encodes into bit-plane rows
    (2, 2, 8, 700, 64, 32, 40, 0, 3),
    (1, 2, 8, 300, 32, 8, 20, 0, 3),
    # physical 2-bit V codes
    (2, 2, 8, 700, 64, 32, 40, 0, 2),
    (1, 2, 8, 300, 32, 8, 20, 0, 2),
])
def test_graph_step_matches_eager(B, Hkv, Hq, T, sk, sv, steps, headroom, v_pack):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache, DecodeGraph, chronoquant_sdpa
    dev = torch.device("cuda")
    K, V = O.ar1_kv(B, Hkv, T + steps, 128, seed=T)
    K = torch.from_numpy(K).to(dev).half()
    V = torch.from_numpy(V).to(dev).half()
    kw = dict(stride_k=sk, stride_v=sv, dead_zone_v=0.0, max_tokens=T + steps + headroom + 8)
    if v_pack < 4:
        kw.update(delta_bits_v=v_pack, v_pack=v_pack)
    eager, graphed = ChronoQuantCache(**kw), ChronoQuantCache(**kw)
    for c in (eager, graphed):
        c.update_and_fetch(K[:, :, :T], V[:, :, :T])
    scale = 1.0 / math.sqrt(128)
    g = DecodeGraph(graphed, Hq, scale, q_dtype=torch.bfloat16, max_len=T + steps + headroom)
    gen = torch.Generator(device="cpu").manual_seed(5)
    for i in range(steps):
        q = (torch.randn((B, Hq, 1, 128), generator=gen) / math.sqrt(128)).to(torch.bfloat16).to(dev)
        k1, v1 = K[:, :, T + i:T + i + 1], V[:, :, T + i:T + i + 1]
        eager.update_and_fetch(k1, v1)
        ref = chronoquant_sdpa(q, None, None, eager, scale)
        out = g.step(k1, v1, q)
        assert graphed.offset == eager.offset == T + i + 1
        _close(out, ref)
    torch.cuda.synchronize()
    assert int(g.len[0]) == T + steps and int(g.len[1]) == 0
    for a, b in zip(eager.state, graphed.state):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    assert torch.equal(eager.store.buf, graphed.store.buf)  # the physical pages too
    if headroom == 0:
        k1, v1 = K[:, :, :1], V[:, :, :1]
        with pytest.raises(ValueError):
            g.step(k1, v1, torch.zeros((B, Hq, 1, 128), dtype=torch.bfloat16, device=dev))  # past max_len


@pytest.mark.gpu
def test_double_buffered_graph_matches_single():
    """buffers=2: two captured graphs over alternating input/output sets, fed
    from pinned host memory on a copy stream while the previous step runs
    (the serving loop of bench.py's e2e), give bit-identical outputs and
    cache bytes to the one-buffer graph stepping the same tokens."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache, DecodeGraph
    dev = torch.device("cuda")
    B, Hkv, Hq, T, steps = 2, 2, 8, 700, 24
    K, V = O.ar1_kv(B, Hkv, T + steps, 128, seed=11)
    K = torch.from_numpy(K).to(dev).half()
    V = torch.from_numpy(V).to(dev).half()
    kw = dict(stride_k=64, stride_v=32, delta_bits_v=3, max_tokens=T + steps + 8)
    one, two = ChronoQuantCache(**kw), ChronoQuantCache(**kw)
    for c in (one, two):
        c.update_and_fetch(K[:, :, :T], V[:, :, :T])
    scale = 1.0 / math.sqrt(128)
    g1 = DecodeGraph(one, Hq, scale, q_dtype=torch.bfloat16, max_len=T + steps)
    g2 = DecodeGraph(two, Hq, scale, q_dtype=torch.bfloat16, max_len=T + steps, buffers=2)
    assert g2.buffers == 2 and g2.inputs_of(0).data_ptr() != g2.inputs_of(1).data_ptr()
    gen = torch.Generator(device="cpu").manual_seed(3)
    qs = [(torch.randn((B, Hq, 1, 128), generator=gen) / math.sqrt(128)).to(torch.bfloat16) for _ in range(steps)]
    # each step's flat input row (K | V | q bytes), pinned on the host
    rows = []
    for i in range(steps):
        g1.keys.copy_(K[:, :, T + i:T + i + 1])
        g1.values.copy_(V[:, :, T + i:T + i + 1])
        g1.queries.copy_(qs[i].to(dev))
        rows.append(g1.inputs.cpu().clone())
    hin = torch.stack(rows).pin_memory()
    ref = []
    for i in range(steps):
        g1.inputs.copy_(hin[i].to(dev))
        ref.append(g1.replay().clone())
    copy = torch.cuda.Stream(dev)
    main = torch.cuda.current_stream()
    ev_in, ev_done, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    houts = [torch.empty((B, Hq, 1, 128), dtype=torch.bfloat16).pin_memory() for _ in range(steps)]

    def h2d(k):
        s = k % 2
        with torch.cuda.stream(copy):
            if k >= 2:
                copy.wait_event(ev_done[s])
            g2.inputs_of(s).copy_(hin[k], non_blocking=True)
            ev_in[s].record(copy)

    h2d(0)
    for k in range(steps):
        s = k % 2
        if k + 1 < steps:
            h2d(k + 1)
        main.wait_event(ev_in[s])
        if k >= 2:
            main.wait_event(ev_out[s])
        out = g2.replay()
        assert out.data_ptr() == g2.out_of(s).data_ptr()
        ev_done[s].record(main)
        with torch.cuda.stream(copy):
            copy.wait_event(ev_done[s])
            houts[k].copy_(out, non_blocking=True)
            ev_out[s].record(copy)
    torch.cuda.synchronize()
    for k in range(steps):
        assert torch.equal(houts[k], ref[k].cpu()), k
    for a, b in zip(one.state, two.state):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
