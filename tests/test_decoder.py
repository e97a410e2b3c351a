"""The end-to-end decoder (BASELINE config 5's shape, here shrunk): one greedy
decode step as a CUDA-graph replay, through the compressed caches.

Bars: graph replays give logits within 1e-3 relative (L2) of the same decoder
stepped eagerly with the same kernels; both are within 2e-2 relative of a decoder
with the same weights and context whose attention is a plain PyTorch fp32
reference (softmax(q k^T scale) v over each layer cache's fp16 reconstruction,
cache.py:131-160), fed the same input ids.  The 2e-2 covers bf16 activations
carrying per-layer differences through the network to the logits, plus the
decode kernel dequantising in fp32 (the fused path, kernels.py:152-155) where
the reference rounds the reconstruction to fp16; the attention kernels' own
bars are in test_gpu_parity.py."""

import math

import pytest
import torch

from chronoquant_mlx_b200.decoder import DecoderConfig, Qwen3StyleDecoder

pytestmark = pytest.mark.gpu

CFG = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1000)


def _reference_attention(dec):
    def attend(L, q, k, v):
        cache = L["cache"]
        cache.update_and_fetch(k.unsqueeze(2), v.unsqueeze(2))
        kk, vv = cache.reconstruct_history()
        rep = q.shape[1] // kk.shape[1]
        kk = kk.float().repeat_interleave(rep, 1)
        vv = vv.float().repeat_interleave(rep, 1)
        s = torch.einsum("bhd,bhtd->bht", q.float(), kk) / math.sqrt(q.shape[-1])
        return torch.einsum("bht,bhtd->bhd", torch.softmax(s, -1), vv).to(q.dtype)
    return attend


@pytest.mark.parametrize("cache_kwargs", [dict(), dict(stride_k=64, stride_v=32, delta_bits_v=3, dead_zone_v=0.05)])
def test_graph_decode_matches_eager_and_reference(cache_kwargs):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    B, T0, steps = 2, 300, 4
    g = Qwen3StyleDecoder(CFG, B, T0 + steps + 4, cache_kwargs, seed=3)
    e = Qwen3StyleDecoder(CFG, B, T0 + steps + 4, cache_kwargs, seed=3)
    r = Qwen3StyleDecoder(CFG, B, T0 + steps + 4, cache_kwargs, seed=3)
    for d in (g, e, r):
        d.fill_context(T0)
        d.ids.copy_(torch.tensor([5, 77], device="cuda"))
    g.capture()
    ref_attn = _reference_attention(r)
    for _ in range(steps):
        ids = r.ids.clone()
        g.ids.copy_(ids)
        e.ids.copy_(ids)
        lg = g.decode(1).float().clone()
        le = e.step_eager().float()
        lr = r.step_eager(ref_attn).float()
        assert (lg - le).norm() <= 1e-3 * le.norm()  # same kernels; cuBLAS may pick other algorithms in a graph
        assert torch.isfinite(lg).all()
        rel = (lg - lr).norm() / lr.norm()
        assert rel < 2e-2, float(rel)
    assert g.layers[0]["cache"].offset == T0 + steps == r.layers[1]["cache"].offset
    assert int(g.layers[1]["len"][0]) == T0 + steps
    # layer 0's new K/V depend only on the ids and weights: the fused step encodes them exactly as
    # update_and_fetch does (deeper layers see slightly different attention outputs)
    for x, y in zip(g.layers[0]["cache"].state, r.layers[0]["cache"].state):
        assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
