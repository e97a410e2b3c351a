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
@pytest.mark.parametrize("B,Hkv,Hq,T,sk,sv,steps,headroom", [
    (2, 2, 8, 500, 32, 8, 40, 0),     # crosses I-frames of both strides and a chunk boundary
    (1, 4, 16, 1000, 64, 32, 70, 0),  # Full-Throttle strides, crosses a page boundary
    # a graph sized for far more tokens than are cached: the launch has more warps than the
    # current length has chunks, and only as many as there are chunks take work
    (1, 2, 8, 300, 64, 32, 12, 20000),
    (2, 2, 8, 100, 32, 8, 8, 3000),
])
def test_graph_step_matches_eager(B, Hkv, Hq, T, sk, sv, steps, headroom):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import ChronoQuantCache, DecodeGraph, chronoquant_sdpa
    dev = torch.device("cuda")
    K, V = O.ar1_kv(B, Hkv, T + steps, 128, seed=T)
    K = torch.from_numpy(K).to(dev).half()
    V = torch.from_numpy(V).to(dev).half()
    kw = dict(stride_k=sk, stride_v=sv, dead_zone_v=0.0, max_tokens=T + steps + headroom + 8)
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
    if headroom == 0:
        k1, v1 = K[:, :, :1], V[:, :, :1]
        with pytest.raises(ValueError):
            g.step(k1, v1, torch.zeros((B, Hq, 1, 128), dtype=torch.bfloat16, device=dev))  # past max_len
