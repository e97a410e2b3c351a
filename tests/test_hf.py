"""The transformers hook: a tiny random-init Qwen3-style decoder (GQA 4,
head_dim 128) run with ``attn_implementation="chronoquant"`` and a
``ChronoQuantHFCache``, prefill then token-by-token decode.

Bar: logits within 1e-2 relative (L2) of the same model whose attention is a
plain PyTorch fp32 reference of the same op -- softmax(q k^T * scale) v over
the cache's own fp16 reconstruction (cache.py:131-160) -- with the same
compressed cache, so only the attention kernels differ.  The CPU tests check
the cache protocol and the registration without running a model."""

import math

import pytest
import torch

transformers = pytest.importorskip("transformers")

from chronoquant_mlx_b200 import hf


def test_registration_and_protocol_on_cpu():
    hf.register()
    from transformers import AttentionInterface
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    assert AttentionInterface._global_mapping.get(hf.NAME) is hf.chronoquant_attention or \
        hf.NAME in AttentionInterface()
    assert hf.NAME in ALL_MASK_ATTENTION_FUNCTIONS
    cfg = transformers.Qwen3Config(num_hidden_layers=3)
    c = hf.ChronoQuantHFCache(cfg, stride_k=64, stride_v=32)
    assert len(c.layers) == 3 and [x.cq.layer_idx for x in c.layers] == [0, 1, 2]
    assert all(x.cq.stride_k == 64 for x in c.layers)
    assert c.get_seq_length() == 0 and c.layers[1].get_mask_sizes(5) == (5, 0)
    with pytest.raises(NotImplementedError):
        c.layers[0].crop(1)


def _reference_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """fp32 PyTorch attention over the ChronoQuant cache's fp16 reconstruction."""
    cache = getattr(key, hf._TAG)
    k, v = cache.reconstruct_history()
    q = query.float()
    B, Hq, Tq, D = q.shape
    rep = Hq // k.shape[1]
    k = k.float().repeat_interleave(rep, dim=1)
    v = v.float().repeat_interleave(rep, dim=1)
    s = (q * scaling) @ k.transpose(-1, -2)
    T = k.shape[2]
    qi = torch.arange(T - Tq, T, device=q.device)[:, None]
    s = s.masked_fill(qi < torch.arange(T, device=q.device)[None], float("-inf"))
    out = torch.softmax(s, -1) @ v
    return out.to(query.dtype).transpose(1, 2).contiguous(), None


@pytest.mark.gpu
def test_qwen3_style_model_matches_fp32_reference():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    hf.register()
    AttentionInterface.register("cq_reference", _reference_attention)
    AttentionMaskInterface.register("cq_reference", sdpa_mask)
    torch.manual_seed(0)
    cfg = transformers.Qwen3Config(vocab_size=512, hidden_size=1024, intermediate_size=2048, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=4096)
    model = transformers.Qwen3ForCausalLM(cfg).to(torch.float16).cuda().eval()
    ids = torch.randint(0, 512, (2, 300), device="cuda")
    logits = {}
    for impl in (hf.NAME, "cq_reference"):
        model.set_attn_implementation(impl)
        cache = hf.ChronoQuantHFCache(cfg)
        outs = []
        with torch.no_grad():
            outs.append(model(ids[:, :296], past_key_values=cache, use_cache=True).logits[:, -48:].float())
            for t in range(296, 300):  # decode one token at a time
                outs.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits.float())
        assert cache.get_seq_length() == 300 and cache.nbytes > 0
        logits[impl] = torch.cat(outs, 1)
    a, b = logits[hf.NAME], logits["cq_reference"]
    rel = (a - b).norm() / b.norm()
    assert torch.isfinite(a).all() and rel < 1e-2, float(rel)
