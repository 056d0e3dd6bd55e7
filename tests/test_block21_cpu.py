"""Host-side checks of the 2.1 block (no GPU): parameter names against the
reference golden, the modulation vectors of the cached decode, the prefix
segments against the reference's, and that the block refuses CPU tensors
(there is no CPU path)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from qwen_image_accel_b200.optimizations.prefill import prefix_segments
from qwen_image_accel_b200.qwen21 import Block21Config, KVCache, block21_parameter_shapes, modulation_values

GOLD = Path(__file__).resolve().parent / "golden"


def test_parameter_names_match_reference_block():
    g = np.load(GOLD / "block21_tiny.npz")
    dim, heads = g["dims"].tolist()
    assert sorted(block21_parameter_shapes(Block21Config(dim=dim, heads=heads))) == sorted(g["keys"].tolist())


def test_modulation_values_follow_reference_decode_cache():
    """(1 + s1, tanh g1, 1 + s2, tanh g2) of the sampled rows, in bf16
    (src/qwen_image_accel/optimizations/fusion.py:45-49)."""
    torch.manual_seed(0)
    mod = torch.randn(3, 4 * 512).to(torch.bfloat16)
    vals = modulation_values(mod)
    s1, g1, s2, g2 = mod[:-1].chunk(4, dim=-1)
    want = (1 + s1[:, None], g1[:, None].tanh(), 1 + s2[:, None], g2[:, None].tanh())
    for a, b in zip(vals, want):
        assert a.shape == (2, 1, 512) and a.is_contiguous() and torch.equal(a, b)


@pytest.mark.parametrize("name", ["t2i", "edit", "adjacent", "long"])
def test_prefix_segments_match_reference(name):
    d = np.load(GOLD / "block_causal.npz")
    ids = torch.from_numpy(d[f"image_ids_{name}"])
    prefix_len = int((~d[f"target_{name}"]).sum())
    got = np.array([(a, b, int(t)) for a, b, t in prefix_segments(ids, prefix_len)], np.int64).reshape(-1, 3)
    assert np.array_equal(got, d[f"segments_{name}"])


def test_kv_cache_container():
    cache = KVCache(3)
    with pytest.raises(RuntimeError):
        cache.get_layer(1).get()
    k = torch.zeros(1, 4, 2, 128)
    cache.get_layer(1).store(k, k)
    assert cache.get_layer(1).get()[0] is k


def test_interleaved_gate_value_layout():
    from qwen_image_accel_b200.optimizations.mxfp8 import interleaved_gate_value
    g = torch.arange(96 * 4, dtype=torch.float32).view(96, 4)
    v = -g - 1
    s = interleaved_gate_value(g, v)
    assert s.shape == (192, 4)
    for j in range(3):
        assert torch.equal(s[64 * j:64 * j + 32], g[32 * j:32 * j + 32])
        assert torch.equal(s[64 * j + 32:64 * j + 64], v[32 * j:32 * j + 32])
    with pytest.raises(ValueError):
        interleaved_gate_value(g[:40], v[:40])
