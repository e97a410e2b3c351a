"""Host-side logic that needs no GPU: API surface, factories, patch, masks,
byte accounting, page sizing, and the no-CPU-fallback rule."""

import json
import math
import os

import pytest
import torch

import chronoquant_mlx_b200 as cq
from chronoquant_mlx_b200 import base
from chronoquant_mlx_b200.cache import ChronoQuantCache, default_page_tokens, make_causal_mask
from oracle import cq_oracle as O


def test_public_names_match_reference():
    for n in ["ChronoQuantCache", "FULL_THROTTLE_V3_CONFIG", "apply", "apply_patch", "create_chronoquant_caches",
              "create_full_throttle_caches", "chronoquant_sdpa"]:
        assert hasattr(cq, n)
    assert cq.FULL_THROTTLE_V3_CONFIG == {"stride_k": 64, "stride_v": 32, "delta_bits_k": 4, "delta_bits_v": 3,
                                          "dead_zone_k": 0.0, "dead_zone_v": 0.05}
    from chronoquant_mlx_b200.kernels import MAX_FUSED_HEAD_DIM
    from chronoquant_mlx_b200.codec import ChronoQuantCodecMLX
    assert MAX_FUSED_HEAD_DIM == 256 and ChronoQuantCodecMLX(delta_bits=3).half_levels == 4


def test_cache_defaults_mirror_reference():
    c = ChronoQuantCache()
    assert (c.stride_k, c.stride_v, c.delta_bits_k, c.delta_bits_v, c.dead_zone_k, c.dead_zone_v, c.use_fused,
            c.per_layer_v_bits, c.layer_idx, c.offset, c.head_dim) == (32, 8, 4, 4, 0.0, 0.05, True, [], 0, 0, None)
    assert c.codec_k.delta_bits == 4 and c.codec_k.stride == 32
    assert c.empty() and not c.has_previous_state() and not c.is_trimmable()
    assert c.state == [] and c.nbytes == 0
    # meta_state: the reference returns "" (cache.py:257-263); here it carries the configuration
    # (strides, bits, dead zones, ...) so saved caches restore self-described, and "" is accepted
    assert c.meta_state[0] == "chronoquant/1" and "stride_k=32" in c.meta_state
    c.meta_state = ""
    assert c.reconstruct_history() == (None, None)


def test_reference_delta_bits_kwarg_rejected_like_reference():
    with pytest.raises(TypeError):
        ChronoQuantCache(stride_k=4, stride_v=2, delta_bits=4)


@pytest.mark.parametrize("T,s", [(0, 8), (1, 8), (8, 8), (9, 8), (100, 32), (16384, 32), (32768, 64)])
def test_frame_counts(T, s):
    assert ChronoQuantCache._num_keyframes(T, s) == O.num_keyframes(T, s)
    assert ChronoQuantCache._num_pframes(T, s) == O.num_pframes(T, s)


def test_per_token_head_bytes():
    # (256 + (stride-1)*66)/stride per component at D=128
    for s, want in ((32, 71.94), (8, 89.75), (64, 68.97)):
        got = O.active_bytes_per_head(32 * 64 * 4, 128, s) / (32 * 64 * 4)
        assert abs(got - want) < 0.01


def test_page_tokens():
    assert default_page_tokens(32, 8) == 256
    assert default_page_tokens(64, 32) == 256
    assert default_page_tokens(4, 2) == 256
    assert default_page_tokens(3, 5) == 240
    assert default_page_tokens(100, 128) == 3200
    with pytest.raises(ValueError):
        ChronoQuantCache(stride_k=32, stride_v=8, page_tokens=100)


def test_cpu_tensors_rejected_no_fallback():
    c = ChronoQuantCache()
    with pytest.raises(ValueError, match="CUDA"):
        c.update_and_fetch(torch.zeros(1, 2, 3, 128, dtype=torch.float16), torch.zeros(1, 2, 3, 128, dtype=torch.float16))


def test_make_mask():
    assert make_causal_mask(10, 1) is None
    assert make_causal_mask(10, 4) == "causal"
    m = make_causal_mask(10, 4, return_array=True)
    assert m.shape == (4, 10) and bool(m[0, 6]) and not bool(m[0, 7]) and bool(m[3].all())
    w = make_causal_mask(10, 4, window_size=2)
    assert w.shape == (4, 10) and int(w[3].sum()) == 2


class _Other:
    pass


class _Model:
    layers = [0, 1, 2, 3]

    def make_cache(self):
        return [base.KVCache(), base.KVCache(), _Other(), base.KVCache()]


def test_factories_match_reference_fixture(golden_dir):
    meta = json.load(open(os.path.join(golden_dir, "golden_meta.json")))["factories"]
    caches = cq.create_chronoquant_caches(_Model(), per_layer_v_bits=[4, 3, 2])
    for c, ref in zip(caches, meta["create_chronoquant_caches_per_layer_v_bits_4_3_2"]):
        if ref is None:
            assert isinstance(c, _Other)
            continue
        for k in ("stride_k", "stride_v", "delta_bits_k", "delta_bits_v", "dead_zone_k", "dead_zone_v",
                  "use_fused", "per_layer_v_bits", "layer_idx"):
            assert getattr(c, k) == ref[k], k
        assert c._get_codec_for_v().delta_bits == ref["v_codec_bits"]
    ft = cq.create_full_throttle_caches(_Model(), use_fused=False)
    for c, ref in zip(ft, meta["create_full_throttle_caches"]):
        if ref is None:
            continue
        for k, v in ref.items():
            assert getattr(c, k) == v, k


def test_make_prompt_cache_fallback():
    class M:
        layers = [0, 1]
    caches = cq.create_chronoquant_caches(M())
    assert all(isinstance(c, ChronoQuantCache) for c in caches) and caches[1].layer_idx == 1


def test_patch_dispatch_and_revert():
    from chronoquant_mlx_b200 import patch
    orig = base.scaled_dot_product_attention
    cq.apply()
    try:
        assert base.scaled_dot_product_attention is patch._patched_sdpa
        cq.apply_patch()  # idempotent
        # a plain cache reaches the original attention (torch SDPA, CPU is fine here)
        q = torch.randn(1, 4, 1, 16)
        k = torch.randn(1, 2, 5, 16)
        out = base.scaled_dot_product_attention(q, k, k, base.KVCache(), 0.25, None)
        ref = orig(q, k, k, base.KVCache(), 0.25, None)
        assert torch.allclose(out, ref)
    finally:
        patch.revert()
    assert base.scaled_dot_product_attention is orig


def test_kv_cache_and_original_sdpa_causal():
    c = base.KVCache()
    k = torch.randn(1, 2, 6, 8)
    c.update_and_fetch(k[:, :, :4], k[:, :, :4])
    kk, vv = c.update_and_fetch(k[:, :, 4:], k[:, :, 4:])
    assert kk.shape[2] == 6 and c.offset == 6 and c.make_mask(2) == "causal"
    q = torch.randn(1, 2, 2, 8)
    out = base.scaled_dot_product_attention(q, kk, vv, c, 1.0, "causal")
    m = base.create_causal_mask(2, 4)
    ref = torch.nn.functional.scaled_dot_product_attention(q, kk, vv, attn_mask=m, scale=1.0)
    assert torch.allclose(out, ref)
