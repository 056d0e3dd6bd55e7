"""configure_pipeline on a real Diffusers Qwen-Image 2.1 transformer (the
pinned wheel, installed under baseline/_ref): every fused profile routes the
model's decode to libqia_b200.so and the model still matches the Diffusers
golden (tests/golden/model21_tiny.npz: the same 2-block, dim-512 model with
the same seeded weights, run eagerly in bf16 on the CPU by Diffusers itself):
the prefill with kv_cache_mode="extract", then a cached step with new target
latents, by PSNR and cosine at the gates of test_model21_gpu.py.

The reference's default skip list ("0,31") keeps block 0 of the two in bf16,
so the MXFP8 profiles run one bf16 and one MXFP8 block; a second case
quantizes both."""
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import diffusers_ref

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _needs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not diffusers_ref.available():
        pytest.skip("the pinned Diffusers wheel is not installed under baseline/_ref")


def t_bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def psnr(a, ref):
    a, ref = a.double(), ref.double()
    mse = (a - ref).pow(2).mean()
    peak = ref.max() - ref.min()
    return (10 * torch.log10(peak * peak / mse)).item()


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


def tiny_pipe():
    from qwen_image_accel_b200.mmdit import init_parameter
    t21 = diffusers_ref.qwen21()
    model = t21.QwenImage21Transformer2DModel(num_layers=2, num_attention_heads=4, context_in_dim=256)
    model = model.to(torch.bfloat16)
    sd = model.state_dict()
    model.load_state_dict({n: init_parameter(n, tuple(t.shape), seed=13) for n, t in sd.items()})
    model.eval()
    return SimpleNamespace(transformer=model), t21


def run_golden_case(pipe, t21, steps=1):
    g = np.load(GOLD / "model21_tiny.npz")
    lat, lat2, enc = (t_bf16(g[n]).cuda() for n in ("lat", "lat2", "enc"))
    img_mask = torch.from_numpy(g["img_mask"]).cuda()
    shapes = [[tuple(int(v) for v in s) for s in g["shapes"]]]
    cache = t21.QwenImage21KVCache(2)
    model = pipe.transformer
    with torch.no_grad():
        pre = model(hidden_states=lat, encoder_hidden_states=enc, timestep=torch.tensor([0.8], device="cuda"),
                    img_shapes=shapes, img_mask=img_mask, kv_cache=cache, kv_cache_mode="extract",
                    return_dict=False)[0].float().cpu()
        decs = [model(hidden_states=lat2, encoder_hidden_states=enc, timestep=torch.tensor([0.6], device="cuda"),
                      img_shapes=shapes, img_mask=img_mask, kv_cache=cache, kv_cache_mode="cached",
                      return_dict=False)[0].float().cpu() for _ in range(steps)]
    figures = {"prefill": (pre, t_bf16(g["out_prefill"]).float()),
               "cached_k0": (cache.get_layer(0).k.float().cpu(), t_bf16(g["cached_k0"]).float()),
               "cached_step": (decs[-1], t_bf16(g["out_cached"]).float())}
    return figures, decs


# gates of test_model21_gpu.py (measured there: fused 61.7-85.7 dB, mxfp8_sage 46.1-63.6 dB)
CASES = [("fused", None, 55.0, 0.99995), ("graph", None, 55.0, 0.99995), ("fused_sage", None, 40.0, 0.999),
         ("mxfp8", None, 40.0, 0.999), ("mxfp8_sage", None, 40.0, 0.999), ("mxfp8_sage", "", 40.0, 0.999),
         ("mxfp8_balanced_sage", None, 40.0, 0.999)]


@pytest.mark.parametrize("profile,skip,min_psnr,min_cos", CASES,
                         ids=[f"{c[0]}-skip{c[1]!r}" for c in CASES])
def test_profile_on_diffusers_model(profile, skip, min_psnr, min_cos, monkeypatch):
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.pipeline import configure_pipeline
    from qwen_image_accel_b200.profiles import get_profile
    if skip is not None:
        monkeypatch.setenv("QW21_MXFP8_SKIP_BLOCKS", skip)
    pipe, t21 = tiny_pipe()
    config = configure_pipeline(pipe, profile)
    prof = get_profile(profile)
    assert config["profile"] == profile and pipe._qw_optimization is config
    assert config["cuda_graph"] == prof.graph
    if prof.quantized:
        # 7 block linears (q, k, v, out, gate, value, down) per quantized block
        expect = {None: 7, "": 14}[skip] if profile == "mxfp8_sage" or profile == "mxfp8" else 0
        assert config["mxfp8_linears"] == expect, config
    assert hasattr(pipe.transformer, "_qia_decode")
    _lib.launch_count = 0
    steps = 3 if prof.graph else 1
    figures, decs = run_golden_case(pipe, t21, steps=steps)
    assert _lib.launch_count > 0, "the decode did not reach libqia_b200.so"
    if prof.graph:
        assert len(pipe.transformer._qw_graphs) == 1
        assert torch.equal(decs[0], decs[1]) and torch.equal(decs[1], decs[2]), "graph replay differs from capture"
    report = {k: (round(psnr(a, b), 2), round(cosine(a, b), 6)) for k, (a, b) in figures.items()}
    print(profile, skip, report)
    for name, (a, b) in figures.items():
        assert a.shape == b.shape and torch.isfinite(a).all(), name
    for name, (pv, cv) in report.items():
        assert pv >= min_psnr and cv >= min_cos, (name, pv, cv)


def test_graph_replay_equals_eager_decode():
    """The `graph` profile's replayed decode is bit-identical to the same
    routed decode run eagerly (the `fused` profile on an identical model)."""
    from qwen_image_accel_b200.pipeline import configure_pipeline
    outs = {}
    for profile in ("fused", "graph"):
        pipe, t21 = tiny_pipe()
        configure_pipeline(pipe, profile)
        figures, decs = run_golden_case(pipe, t21, steps=2)
        outs[profile] = decs
    assert torch.equal(outs["fused"][-1], outs["graph"][-1])
    assert torch.equal(outs["graph"][0], outs["graph"][1])


def test_configure_twice_and_unknown_profile():
    from qwen_image_accel_b200.pipeline import configure_pipeline
    pipe, _ = tiny_pipe()
    with pytest.raises(ValueError):
        configure_pipeline(pipe, "no_such_profile")
    with pytest.raises(ValueError):
        configure_pipeline(pipe, "fp8_sage")          # retired name
    assert not hasattr(pipe, "_qw_optimization")   # nothing changed before the checks
    configure_pipeline(pipe, "fused")
    with pytest.raises(RuntimeError):
        configure_pipeline(pipe, "mxfp8_sage")


def test_non_bf16_transformer_rejected_before_any_change():
    from qwen_image_accel_b200.pipeline import configure_pipeline
    pipe, _ = tiny_pipe()
    pipe.transformer.to(torch.float32)
    with pytest.raises(ValueError):
        configure_pipeline(pipe, "mxfp8_sage")
    assert not hasattr(pipe, "_qw_optimization")
    assert not hasattr(pipe.transformer, "_qia_decode")
    assert next(pipe.transformer.parameters()).device.type == "cpu"
