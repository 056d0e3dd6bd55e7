"""Multi-step accuracy gate: final latents of a flow-match Euler denoise with
true CFG at the BASELINE dims (D 3072, 24 x 128 heads, text 3584, 1024^2:
4096 image + 256 text tokens, CFG batch 2, seed 42), with the block count
reduced, against the reference's `mxfp8_sage` composition on the Diffusers
v1 MMDiT (oracle/reference_v1.py: torch._scaled_mm MXFP8 linears, the built
SageAttention, blocks 0 and 31 in bf16, the pipeline's CFG and Euler step).
North-star gate: PSNR >= 35 dB on the final latents."""
import pytest
import torch

from oracle import diffusers_ref, reference_v1, sage_ref

pytestmark = pytest.mark.gpu
GRID = (1, 64, 64)


@pytest.fixture(autouse=True)
def _needs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not diffusers_ref.available() or not sage_ref.available():
        pytest.skip("needs the pinned Diffusers (baseline/_ref) and the built SageAttention (oracle/_ref)")


def psnr(a, ref):
    a, ref = a.double(), ref.double()
    mse = (a - ref).pow(2).mean()
    peak = ref.max() - ref.min()
    return (10 * torch.log10(peak * peak / mse)).item()


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


@pytest.mark.parametrize("layers,sigmas", [(4, [1.0, 0.9, 0.75, 0.5, 0.25]),
                                           (2, [1.0 - i / 40 for i in range(41)])],
                         ids=["4blocks-4steps", "2blocks-40steps"])
def test_final_latents_vs_reference_mxfp8_sage(layers, sigmas):
    from qwen_image_accel_b200.mmdit import MMDiT, MMDiTConfig, random_parameters
    g = torch.Generator(device="cuda").manual_seed(42)
    lat = torch.randn(1, GRID[1] * GRID[2], 64, device="cuda", dtype=torch.bfloat16, generator=g)
    pe = torch.randn(1, 256, 3584, device="cuda", dtype=torch.bfloat16, generator=g)
    ne = torch.randn(1, 256, 3584, device="cuda", dtype=torch.bfloat16, generator=g)
    ref_model = reference_v1.build(layers, seed=42)
    try:
        ref = reference_v1.denoise(ref_model, lat, pe, ne, sigmas, GRID).float().cpu()
    finally:
        ref_model._qia_restore()
    del ref_model
    torch.cuda.empty_cache()
    cfg = MMDiTConfig(num_layers=layers)
    # the seeded recipe is reproducible per device type: draw on the CPU, as reference_v1.build does
    model = MMDiT(cfg, random_parameters(cfg, 42, "cpu"), device="cuda", profile="mxfp8_sage")
    assert model.skip_blocks == {0, 31} and not model.blocks[0].quantized and model.blocks[1].quantized
    x = lat
    for i in range(len(sigmas) - 1):
        x = model.denoise_step(x, pe, ne, sigmas[i], sigmas[i + 1], GRID)
    mine = x.float().cpu()
    p, c = psnr(mine, ref), cosine(mine, ref)
    print(f"{layers} blocks, {len(sigmas) - 1} steps: final latents PSNR {p:.2f} dB, cosine {c:.6f} "
          "vs the reference mxfp8_sage composition")
    assert torch.isfinite(mine).all()
    assert p >= 35.0 and c >= 0.995     # north star: PSNR >= 35 dB (measured 42.8 / 54.7 dB)
