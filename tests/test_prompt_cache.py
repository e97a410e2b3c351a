"""Saving and restoring caches: meta_state carries the configuration; a
prompt-cache file (mlx_lm's safetensors layout) holds each layer's reference-
layout state.  Bars: configuration round trip exact; restored states
bit-identical; attention over a restored cache identical to the original."""

import math

import numpy as np
import pytest
import torch

from chronoquant_mlx_b200 import ChronoQuantCache, FULL_THROTTLE_V3_CONFIG, load_prompt_cache, save_prompt_cache
from oracle import cq_oracle as O


def test_meta_state_configures_an_empty_cache():
    a = ChronoQuantCache(**FULL_THROTTLE_V3_CONFIG, layer_idx=3)
    b = ChronoQuantCache()
    b.meta_state = a.meta_state
    for k in ChronoQuantCache._META_KEYS:
        assert getattr(a, k) == getattr(b, k), k
    assert b.meta_state == a.meta_state
    c = ChronoQuantCache(stride_k=16)
    c.meta_state = ""  # the reference's meta_state: keep the constructor's configuration
    assert c.stride_k == 16
    with pytest.raises(ValueError):
        c.meta_state = ("not-chronoquant",)


def test_per_layer_v_bits_survive_meta_state():
    a = ChronoQuantCache(per_layer_v_bits=[4, 3, 2], layer_idx=1)
    b = ChronoQuantCache()
    b.meta_state = a.meta_state
    assert b.per_layer_v_bits == [4, 3, 2] and b.layer_idx == 1
    assert b._get_codec_for_v().delta_bits == 3


def test_file_of_empty_caches_round_trips(tmp_path):
    f = str(tmp_path / "empty.safetensors")
    save_prompt_cache(f, [ChronoQuantCache(stride_k=64, stride_v=32), ChronoQuantCache()], {"model": "x"})
    caches, meta = load_prompt_cache(f, return_metadata=True, device="cpu")
    assert meta == {"model": "x"}
    assert [c.stride_k for c in caches] == [64, 32] and all(c.offset == 0 for c in caches)


@pytest.mark.gpu
def test_saved_caches_restore_bit_exact(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chronoquant_mlx_b200 import chronoquant_sdpa
    layers = []
    for i, kw in enumerate([dict(), FULL_THROTTLE_V3_CONFIG, dict(per_layer_v_bits=[4, 3], layer_idx=1)]):
        K, V = O.ar1_kv(2, 2, 333, 128, seed=40 + i)
        c = ChronoQuantCache(**kw)
        c.update_and_fetch(torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda())
        layers.append(c)
    f = str(tmp_path / "caches.safetensors")
    save_prompt_cache(f, layers, {"tokens": "333"})
    restored, meta = load_prompt_cache(f, return_metadata=True)
    assert meta == {"tokens": "333"}
    q = (torch.randn(2, 8, 1, 128) / math.sqrt(128)).to(torch.float16).cuda()
    for a, b in zip(layers, restored):
        assert b.meta_state == a.meta_state and b.offset == a.offset and b.nbytes == a.nbytes
        for x, y in zip(a.state, b.state):
            assert x.dtype == y.dtype and x.shape == y.shape
            assert torch.equal(x.view(torch.uint8), y.view(torch.uint8))
        oa = chronoquant_sdpa(q, None, None, a, 1 / math.sqrt(128))
        ob = chronoquant_sdpa(q, None, None, b, 1 / math.sqrt(128))
        assert torch.equal(oa, ob)
