"""The 2.1 block-causal prefill mask on the CPU, pinned to the reference.

tests/golden/block_causal.npz holds, for four sequence layouts, the token
metadata, the prefix segments and the dense mask of the flex mask_mod, all
produced by the pinned Diffusers wheel (tests/golden/make_golden.py). Checked
here, bit-exact (integer work):
* the oracle's dense restatement of mask_mod against the golden mask;
* the per-query key limits (oracle loop and the package's on-device torch
  form) against the golden mask and against the golden segments;
* the key compaction used for padded prompts: every query sees the same set
  of original keys as in the golden mask;
* the masked Sage oracle: with every limit at Skv it is the unmasked oracle,
  and it stays within the Sage cosine gate of exact masked attention.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from qwen_image_accel_b200.optimizations.prefill import block_causal_kv_limits, compact_valid_keys

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "block_causal.npz")
LAYOUTS = ["t2i", "edit", "adjacent", "long"]


@pytest.mark.parametrize("name", LAYOUTS)
def test_oracle_mask_matches_reference_mask_mod(name):
    got = oracle.block_causal_mask(GOLD[f"image_ids_{name}"], GOLD[f"key_valid_{name}"])
    assert np.array_equal(got, GOLD[f"mask_{name}"])


@pytest.mark.parametrize("name", LAYOUTS)
def test_kv_limits_reproduce_reference_mask(name):
    ids = GOLD[f"image_ids_{name}"]
    s = ids.shape[0]
    lim = oracle.block_causal_kv_limits(ids)
    dense = np.arange(s)[None, :] < lim[:, None]
    # batch row 0 of the golden has every key valid
    assert GOLD[f"key_valid_{name}"][0].all()
    assert np.array_equal(dense, GOLD[f"mask_{name}"][0])
    mine = block_causal_kv_limits(torch.from_numpy(ids)).numpy()
    assert mine.dtype == np.int32 and np.array_equal(mine, lim)


@pytest.mark.parametrize("name", LAYOUTS)
def test_kv_limits_follow_reference_segments(name):
    """Every prefix segment sees keys [0, end) (text: its causal triangle),
    the target image every key (transformer_qwenimage21.py:502-541)."""
    ids = GOLD[f"image_ids_{name}"]
    s = ids.shape[0]
    lim = oracle.block_causal_kv_limits(ids)
    segs = GOLD[f"segments_{name}"]
    prefix_len = int((~GOLD[f"target_{name}"]).sum())
    assert segs[-1, 1] == prefix_len
    for start, end, is_text in segs:
        want = np.arange(start, end) + 1 if is_text else np.full(end - start, end)
        assert np.array_equal(lim[start:end], want)
    assert (lim[prefix_len:] == s).all()


@pytest.mark.parametrize("name", LAYOUTS)
def test_key_compaction_keeps_each_querys_key_set(name):
    ids = torch.from_numpy(GOLD[f"image_ids_{name}"])
    kv = torch.from_numpy(GOLD[f"key_valid_{name}"])
    mask = GOLD[f"mask_{name}"]
    b, s = kv.shape
    # keys carry their own index, so the compacted order can be read back
    k = torch.arange(s, dtype=torch.float32)[None, :, None, None].expand(b, s, 1, 1).contiguous()
    kc, vc, lim = compact_valid_keys(k, k.clone(), kv, block_causal_kv_limits(ids))
    assert lim.shape == (b, s) and lim.dtype == torch.int32
    for bi in range(b):
        order = kc[bi, :, 0, 0].long().numpy()
        assert np.array_equal(order, vc[bi, :, 0, 0].long().numpy())
        for qi in range(s):
            seen = set(order[: int(lim[bi, qi])].tolist())
            assert seen == set(np.nonzero(mask[bi, qi])[0].tolist()), (bi, qi)


def test_masked_sage_oracle():
    rng = np.random.default_rng(5)
    ids = GOLD["image_ids_long"]
    s, h = ids.shape[0], 2
    q, k, v = (rng.standard_normal((1, s, h, 128)).astype(np.float32) for _ in range(3))
    full = np.full((1, s), s, np.int32)
    assert np.array_equal(oracle.sage_attention(q, k, v, kv_limit=full), oracle.sage_attention(q, k, v))
    lim = oracle.block_causal_kv_limits(ids)
    got = oracle.sage_attention(q, k, v, kv_limit=lim)
    exact = oracle.attention_fp32(q, k, v, mask=oracle.block_causal_mask(ids))
    cos = float((got.ravel() @ exact.ravel()) / (np.linalg.norm(got) * np.linalg.norm(exact)))
    assert cos >= 0.999
    # the first text row sees only itself: its output is its own value row
    assert np.allclose(exact[0, 0], v[0, 0], atol=1e-6)
    zero = oracle.sage_attention(q, k, v, kv_limit=np.zeros(s, np.int32))
    assert np.array_equal(zero, np.zeros_like(zero))
