"""Model-level CPU checks: the v1 MMDiT names, RoPE tables and the eager CPU
restatement (oracle/mmdit_cpu.py) against the Diffusers golden."""
from pathlib import Path

import numpy as np
import torch

GOLD = Path(__file__).resolve().parent / "golden"


def t_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def tiny():
    from qwen_image_accel_b200.mmdit import MMDiTConfig
    return MMDiTConfig(num_layers=2, num_attention_heads=4, joint_attention_dim=512)


def test_parameter_names_match_diffusers():
    from qwen_image_accel_b200.mmdit import parameter_shapes
    g = np.load(GOLD / "mmdit_tiny.npz")
    assert sorted(parameter_shapes(tiny())) == sorted(g["keys"].tolist())


def test_rope_tables_match_diffusers():
    from qwen_image_accel_b200.mmdit import rope_tables
    g = np.load(GOLD / "rope_rms.npz")
    img, txt = rope_tables(1, 4, 4, 16)
    assert np.array_equal(torch.view_as_real(img).numpy(), g["img_freqs"])
    assert np.array_equal(torch.view_as_real(txt).numpy(), g["txt_freqs"])
    m = np.load(GOLD / "mmdit_tiny.npz")
    f, h, w, lt = m["shape"].tolist()
    img, txt = rope_tables(f, h, w, lt)
    assert np.array_equal(torch.view_as_real(img).numpy(), m["img_freqs"])
    assert np.array_equal(torch.view_as_real(txt).numpy(), m["txt_freqs"])


def test_cpu_restatement_matches_diffusers_golden():
    from oracle import mmdit_cpu
    from qwen_image_accel_b200.mmdit import parameter_shapes, init_parameter, rope_tables
    cfg = tiny()
    g = np.load(GOLD / "mmdit_tiny.npz")
    shapes = parameter_shapes(cfg)
    p = {n: init_parameter(n, s, seed=7) for n, s in shapes.items()}
    f, h, w, lt = g["shape"].tolist()
    img, txt = rope_tables(f, h, w, lt)
    out = mmdit_cpu.model_forward(p, cfg, t_bf16(g["x"]), t_bf16(g["enc"]), torch.tensor([0.7, 0.7]), img, txt)
    ref = t_bf16(g["out"]).float()
    err = (out.float() - ref).norm() / ref.norm()
    assert err < 1e-2, err
