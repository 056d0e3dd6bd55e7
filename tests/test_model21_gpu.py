"""The whole Qwen-Image 2.1 transformer on the sm_100a kernels
(qwen21_model.Qwen21Transformer) against the Diffusers
QwenImage21Transformer2DModel golden (tests/golden/model21_tiny.npz: 2 blocks,
dim 512, a condition-image edit in the vision-language slot layout): the
prefill with kv_cache_mode="extract" (whole joint sequence, layer 0's
extracted K), then a cached step with new target latents, by PSNR and cosine
per profile (printed)."""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


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


# measured on B200: fused 61.7-85.7 dB (cosine >= 0.999987), mxfp8_sage 46.1-63.6 dB (cosine >= 0.99929)
@pytest.mark.parametrize("profile,sage_prefill,min_psnr,min_cos",
                         [("fused", False, 55.0, 0.99995), ("mxfp8_sage", False, 40.0, 0.999),
                          ("mxfp8_sage", True, 40.0, 0.999)])
def test_prefill_extract_then_cached_step(profile, sage_prefill, min_psnr, min_cos):
    from qwen_image_accel_b200.mmdit import init_parameter
    from qwen_image_accel_b200.qwen21 import Block21Config, KVCache
    from qwen_image_accel_b200.qwen21_model import Qwen21Transformer, model21_parameter_shapes
    g = np.load(GOLD / "model21_tiny.npz")
    cfg = Block21Config(dim=512, heads=4)
    shapes = model21_parameter_shapes(2, cfg, context_in_dim=256)
    model = Qwen21Transformer(lambda n: init_parameter(n, shapes[n], seed=13), num_layers=2, cfg=cfg,
                              context_in_dim=256, device="cuda", profile=profile, sage_prefill=sage_prefill)
    lat, lat2, enc = (t_bf16(g[n]).cuda() for n in ("lat", "lat2", "enc"))
    img_mask = torch.from_numpy(g["img_mask"]).cuda()
    img_shapes = [[tuple(int(v) for v in s) for s in g["shapes"]]]
    cache = KVCache(2)
    out_pre = model.forward(lat, enc, torch.tensor([0.8], device="cuda"), img_shapes, img_mask, kv_cache=cache,
                            kv_cache_mode="extract").float().cpu()
    out_dec = model.forward(lat2, enc, torch.tensor([0.6], device="cuda"), img_shapes, img_mask, kv_cache=cache,
                            kv_cache_mode="cached").float().cpu()
    figures = {"prefill": (out_pre, t_bf16(g["out_prefill"]).float()),
               "cached_k0": (cache.get_layer(0).k.float().cpu(), t_bf16(g["cached_k0"]).float()),
               "cached_step": (out_dec, t_bf16(g["out_cached"]).float())}
    report = {k: (round(psnr(a, b), 2), round(cosine(a, b), 6)) for k, (a, b) in figures.items()}
    print(profile, "sage_prefill" if sage_prefill else "sdpa_prefill", report)
    for name, (a, b) in figures.items():
        assert a.shape == b.shape and torch.isfinite(a).all(), name
    for name, (pv, cv) in report.items():
        assert pv >= min_psnr and cv >= min_cos, (name, pv, cv)


ROPE_LAYOUTS = {
    "golden": ([("t", 20), ("i", 48), ("t", 6), ("i", 64)], [(1, 6, 8), (1, 8, 8)]),
    "adjacent": ([("t", 4), ("i", 4), ("i", 6), ("t", 2), ("i", 12)], [(1, 2, 2), (1, 2, 3), (1, 3, 4)]),
    "edit_1024": ([("t", 113), ("i", 4096), ("t", 20), ("i", 4096)], [(1, 64, 64), (1, 64, 64)]),
    "t2i_2048_odd": ([("t", 97), ("i", 128 * 96)], [(1, 128, 96)]),
    "trailing_text": ([("t", 3), ("i", 15), ("t", 300)], [(1, 3, 5)]),
}


@pytest.mark.parametrize("name", list(ROPE_LAYOUTS))
def test_rope_table_on_device_is_bit_identical(name):
    """qia_rope21_table (positions by prefix sums on the GPU, then the exact
    per-axis gather) against the host table of the reference's loop
    (rope_table, itself pinned to QwenImage21Rope's output)."""
    from qwen_image_accel_b200.qwen21_model import rope_table, rope_table_device
    runs, shapes = ROPE_LAYOUTS[name]
    mask = torch.cat([torch.full((n,), kind == "i") for kind, n in runs])
    host = rope_table(shapes, mask)
    dev = rope_table_device(shapes, mask.cuda())
    assert dev.shape == host.shape
    assert torch.equal(torch.view_as_real(dev).cpu(), torch.view_as_real(host))


def test_rope_table_device_rejects_positions_past_the_tables():
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.qwen21_model import rope_table_device
    mask = torch.ones(2 * 4100, dtype=torch.bool, device="cuda")
    with pytest.raises(_lib.QiaError):
        rope_table_device([(1, 2, 4100)], mask)        # a 4100-wide grid needs 2050 negative rows (1024 held)
