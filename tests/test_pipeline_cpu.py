"""The host side of configure_pipeline and the MXFP8 layer selection, on the
CPU: the checks that must fire before a pipeline is changed, and the
QW21_MXFP8_LAYERS / QW21_MXFP8_SKIP_BLOCKS parsing."""
from types import SimpleNamespace

import pytest
import torch

from oracle import diffusers_ref


def test_selected_layers_groups_and_lists():
    from qwen_image_accel_b200.optimizations.mxfp8 import LAYER_GROUPS, selected_layers
    assert selected_layers("all") == set(LAYER_GROUPS["attention"]) | set(LAYER_GROUPS["mlp"])
    assert selected_layers("mlp") == set(LAYER_GROUPS["mlp"])
    assert selected_layers(" attn.to_q , img_mlp.out ,") == {"attn.to_q", "img_mlp.out"}
    with pytest.raises(ValueError):
        selected_layers("attn.to_q,attn.nope")


def test_selected_layers_environment(monkeypatch):
    from qwen_image_accel_b200.optimizations.mxfp8 import selected_layers
    monkeypatch.setenv("QW21_MXFP8_LAYERS", "attention")
    assert "attn.to_out.0" in selected_layers() and "img_mlp.out" not in selected_layers()
    assert selected_layers("mlp") != selected_layers()     # an explicit argument wins


def test_skip_block_indices(monkeypatch):
    from qwen_image_accel_b200.optimizations.mxfp8 import skip_block_indices
    monkeypatch.delenv("QW21_MXFP8_SKIP_BLOCKS", raising=False)
    assert skip_block_indices() == {0, 31}                          # the reference's default
    assert skip_block_indices(None, "0,1,2,29,30,31") == {0, 1, 2, 29, 30, 31}   # a profile's own list
    assert skip_block_indices("") == set()
    assert skip_block_indices([3, 4]) == {3, 4}
    monkeypatch.setenv("QW21_MXFP8_SKIP_BLOCKS", "5")
    assert skip_block_indices() == {5} and skip_block_indices(None, "0,1") == {5}   # the environment wins
    assert skip_block_indices("7") == {7}                           # an explicit argument wins over both


def _pipe():
    if not diffusers_ref.available():
        pytest.skip("the pinned Diffusers wheel is not installed under baseline/_ref")
    t21 = diffusers_ref.qwen21()
    model = t21.QwenImage21Transformer2DModel(num_layers=1, num_attention_heads=2, context_in_dim=128)
    return SimpleNamespace(transformer=model.to(torch.bfloat16))


def test_profile_names_checked_first():
    from qwen_image_accel_b200.pipeline import configure_pipeline
    pipe = _pipe()
    with pytest.raises(ValueError, match="Unknown"):
        configure_pipeline(pipe, "turbo")
    with pytest.raises(ValueError, match="retired"):
        configure_pipeline(pipe, "sage")
    with pytest.raises(NotImplementedError):
        configure_pipeline(pipe, "compiled")
    assert not hasattr(pipe, "_qw_optimization")


def test_fused_profiles_refuse_a_host_without_b200_before_changing_anything():
    if torch.cuda.is_available():
        pytest.skip("checks the refusal on a host without the GPU")
    from qwen_image_accel_b200.pipeline import configure_pipeline
    pipe = _pipe()
    before = {n: p.data_ptr() for n, p in pipe.transformer.named_parameters()}
    for profile in ("fused", "fused_sage", "mxfp8_sage", "graph"):
        with pytest.raises(RuntimeError):
            configure_pipeline(pipe, profile)
    assert not hasattr(pipe, "_qw_optimization") and not hasattr(pipe.transformer, "_qia_decode")
    assert before == {n: p.data_ptr() for n, p in pipe.transformer.named_parameters()}


def test_fused_profiles_refuse_a_float32_transformer():
    from qwen_image_accel_b200.pipeline import configure_pipeline
    pipe = _pipe()
    pipe.transformer.to(torch.float32)
    with pytest.raises(ValueError, match="bf16"):
        configure_pipeline(pipe, "mxfp8_sage")
    assert not hasattr(pipe, "_qw_optimization")
