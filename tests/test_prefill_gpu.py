"""GPU parity of the 2.1 block-causal prefill attention
(qia_sage_attention_prefill through optimizations.prefill).

* with every key limit at Skv the prefill entry is bit-identical to the
  unmasked Sage attention (same quantizers, same kernel, same order);
* on the reference's own golden layouts (tests/golden/block_causal.npz) and
  on a 2.1-sized edit layout: cosine >= 0.999 (the Sage gate) against the
  masked Sage oracle and against exact masked attention, per head;
* padded prompt keys (key_valid) through the key compaction: cosine >= 0.999
  against exact attention under the reference's dense mask;
* a row whose limit is 0 is zero, and bad arguments are rejected.
"""
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "block_causal.npz")


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


def make_qkv(b, s, h, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return tuple(torch.randn(b, s, h, 128, device=DEV, dtype=torch.bfloat16, generator=g) for _ in range(3))


def exact_masked(q, k, v, mask):
    """fp32 SDPA under a bool mask [B or 1, Sq, Skv] of visible keys."""
    qt, kt, vt = (t.float().transpose(1, 2) for t in (q, k, v))
    return F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask[:, None]).transpose(1, 2)


def layout_ids(runs):
    ids, blk = [], 0
    for kind, n in runs:
        ids += [-1] * n if kind == "t" else [blk] * n
        blk += kind == "i"
    return torch.tensor(ids, device=DEV)


def test_full_limits_bit_identical_to_unmasked():
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention, sage_attention_prefill
    q, k, v = make_qkv(2, 700, 3, 11)
    lim = torch.full((700,), 700, device=DEV, dtype=torch.int32)
    assert torch.equal(sage_attention_prefill(q, k, v, lim), sage_attention(q, k, v))
    big = torch.full((2, 700), 10 ** 6, device=DEV, dtype=torch.int32)    # clamped to Skv
    assert torch.equal(sage_attention_prefill(q, k, v, big), sage_attention(q, k, v))


@pytest.mark.parametrize("name", ["t2i", "edit", "adjacent", "long"])
def test_golden_layouts_vs_oracle_and_exact(name):
    from qwen_image_accel_b200.optimizations.prefill import prefill_attention
    ids = torch.from_numpy(GOLD[f"image_ids_{name}"]).to(DEV)
    s, h = ids.shape[0], 2
    q, k, v = make_qkv(1, s, h, 21)
    got = prefill_attention(q, k, v, ids)
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    qf, kf, vf = (t.float().cpu().numpy() for t in (q, k, v))
    lim = oracle.block_causal_kv_limits(GOLD[f"image_ids_{name}"])
    ref = torch.from_numpy(oracle.sage_attention(qf, kf, vf, kv_limit=lim))
    exact = torch.from_numpy(oracle.attention_fp32(qf, kf, vf, mask=oracle.block_causal_mask(ids.cpu().numpy())))
    g = got.float().cpu()
    assert cosine(g, ref) >= 0.999
    assert cosine(g, exact) >= 0.999


def test_edit_layout_2p1_size_per_head():
    """113 text + 1024-token condition image + 20 text + 1024-token target:
    the first query tiles see one or two key tiles, the target every key."""
    from qwen_image_accel_b200.optimizations.prefill import block_causal_kv_limits, prefill_attention
    ids = layout_ids([("t", 113), ("i", 1024), ("t", 20), ("i", 1024)])
    s, h = ids.shape[0], 4
    q, k, v = make_qkv(1, s, h, 31)
    got = prefill_attention(q, k, v, ids).float()
    lim = block_causal_kv_limits(ids)
    mask = (torch.arange(s, device=DEV)[None, :] < lim[:, None])[None]
    ref = exact_masked(q, k, v, mask)
    for hi in range(h):
        assert cosine(got[0, :, hi], ref[0, :, hi]) >= 0.999
    # text rows, where the causal limit cuts inside a tile
    assert cosine(got[0, :113], ref[0, :113]) >= 0.999
    assert cosine(got[0, 1137:1157], ref[0, 1137:1157]) >= 0.999


def test_padded_prompt_keys():
    from qwen_image_accel_b200.optimizations.prefill import prefill_attention
    name = "long"
    ids = torch.from_numpy(GOLD[f"image_ids_{name}"]).to(DEV)
    kv = torch.from_numpy(GOLD[f"key_valid_{name}"]).to(DEV)
    mask = torch.from_numpy(GOLD[f"mask_{name}"]).to(DEV)
    b, s = kv.shape
    q, k, v = make_qkv(b, s, 2, 41)
    got = prefill_attention(q, k, v, ids, key_valid=kv).float()
    ref = exact_masked(q, k, v, mask)
    for bi in range(b):
        assert cosine(got[bi], ref[bi]) >= 0.999


def test_zero_limit_rows_and_batch_limits():
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention_prefill
    q, k, v = make_qkv(2, 300, 2, 51)
    lim = torch.stack([torch.arange(300, device=DEV, dtype=torch.int32),          # row t sees [0, t)
                       torch.full((300,), 300, device=DEV, dtype=torch.int32)])
    got = sage_attention_prefill(q, k, v, lim).float()
    assert torch.isfinite(got).all()
    assert got[0, 0].abs().max().item() == 0.0                                     # limit 0: zeros
    mask = torch.arange(300, device=DEV)[None, None, :] < lim[:, :, None]
    ref = exact_masked(q, k, v, mask)
    assert cosine(got[0, 1:], ref[0, 1:]) >= 0.999
    assert cosine(got[1], ref[1]) >= 0.999


def test_prefill_entry_rejects_bad_arguments():
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention_prefill
    q, k, v = make_qkv(1, 128, 1, 61)
    with pytest.raises(NotImplementedError):
        sage_attention_prefill(q, k, v, torch.zeros(128, device=DEV, dtype=torch.int64))
    with pytest.raises(NotImplementedError):
        sage_attention_prefill(q, k, v, torch.zeros(127, device=DEV, dtype=torch.int32))
    lib = _lib.load()
    import ctypes
    strides = (ctypes.c_int64 * 12)(*([128 * 128, 128, 128] * 4))
    out = torch.empty_like(q)
    rc = lib.qia_sage_attention_prefill(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), None, 0, 1, 128, 128,
                                        1, 128, strides, 0.0, None, 0, None)
    assert rc != 0 and b"kv_limit" in lib.qia_last_error_string()
    assert _lib.device_error() == 0


def test_all_valid_keys_equal_unmasked():
    """key_valid with every key valid leaves the key order and the limits
    unchanged (recounted per sample), so the result is the unmasked call's."""
    from qwen_image_accel_b200.optimizations.prefill import prefill_attention
    ids = torch.from_numpy(GOLD["image_ids_long"]).to(DEV)
    s = ids.shape[0]
    q, k, v = make_qkv(2, s, 2, 71)
    kv = torch.ones(2, s, dtype=torch.bool, device=DEV)
    assert torch.equal(prefill_attention(q, k, v, ids, key_valid=kv), prefill_attention(q, k, v, ids))
