"""Host logic of the whole 2.1 transformer (qwen21_model), bit-exact on the
CPU against the reference's own outputs: the 3-axis RoPE table against
QwenImage21Rope (tests/golden/block21_tiny.npz), the token metadata against
build_token_metadata (tests/golden/block_causal.npz), and the parameter names
against QwenImage21Transformer2DModel's state dict
(tests/golden/model21_tiny.npz)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from qwen_image_accel_b200.qwen21 import Block21Config
from qwen_image_accel_b200.qwen21_model import model21_parameter_shapes, rope_table, token_metadata

GOLD = Path(__file__).resolve().parent / "golden"
# the layouts tests/golden/make_golden.py generated (runs of text / image tokens, image shapes)
LAYOUTS = {
    "t2i": ([("t", 7), ("i", 8)], [(1, 2, 4)]),
    "edit": ([("t", 5), ("i", 6), ("t", 3), ("i", 8)], [(1, 2, 3), (1, 2, 4)]),
    "adjacent": ([("t", 4), ("i", 4), ("i", 6), ("t", 2), ("i", 12)], [(1, 2, 2), (1, 2, 3), (1, 3, 4)]),
    "long": ([("t", 37), ("i", 64), ("t", 11), ("i", 48), ("t", 5), ("i", 96)], [(1, 8, 8), (1, 6, 8), (1, 8, 12)]),
}


def pad_mask(runs):
    return torch.cat([torch.full((n,), kind == "i") for kind, n in runs])


def test_rope_table_matches_reference():
    g = np.load(GOLD / "block21_tiny.npz")
    runs = [("t", 20), ("i", 48), ("t", 6), ("i", 64)]
    got = torch.view_as_real(rope_table([(1, 6, 8), (1, 8, 8)], pad_mask(runs))).numpy()
    assert got.shape == g["rope"].shape and np.array_equal(got, g["rope"])


@pytest.mark.parametrize("name", list(LAYOUTS))
def test_token_metadata_matches_reference(name):
    d = np.load(GOLD / "block_causal.npz")
    runs, shapes = LAYOUTS[name]
    ids, target = token_metadata(pad_mask(runs), shapes)
    assert np.array_equal(ids.numpy(), d[f"image_ids_{name}"]) and np.array_equal(target.numpy(), d[f"target_{name}"])


def test_metadata_rejects_shape_mismatch():
    with pytest.raises(ValueError):
        token_metadata(pad_mask([("t", 3), ("i", 5)]), [(1, 2, 2)])


def test_parameter_names_match_reference_model():
    g = np.load(GOLD / "model21_tiny.npz")
    shapes = model21_parameter_shapes(2, Block21Config(dim=512, heads=4), context_in_dim=256)
    assert sorted(shapes) == sorted(g["keys"].tolist())
