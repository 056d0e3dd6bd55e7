"""GPU parity of the Sage-style attention against the reference's own
SageAttention, built from the pinned tarball (oracle/build_sage_ref.py).

The reference's quantized decode attention is `qw21::sage_decode` ->
sageattn_qk_int8_pv_fp8_cuda(tensor_layout="NHD", qk_quant_gran="per_warp",
pv_accum_dtype="fp32+fp32") (src/qwen_image_accel/optimizations/
sage_attention.py:19-25, SAGE:sageattention/core.py:636-828). Checked here on
the same bf16 inputs:

* Q INT8 codes and per-32-row scales: bit-exact.
* the K smoothing mean: Sage takes it with torch's `k.mean` (core.py:773), a
  float32 sum in torch's reduction order; the kernels here sum in their own
  order, so a mean element can land one bf16 ulp apart when the float32 sum
  sits on a rounding boundary. Every differing element is counted, and must be
  at most 1 ulp and at most 1 in 500 elements.
* K INT8 codes and per-64-row scales: bit-exact when Sage's quantizer is given
  the same mean; against Sage's own mean, every differing code sits in a
  channel whose mean differs, and differs by at most 1.
* V FP8 codes and per-channel scales: bit-exact (Sage's key permutation
  undone).
* the attention output: cosine >= 0.999 against Sage's (the north-star gate)
  and element-wise close.

Inputs follow BASELINE config 3 (B=2, H=24, 256 text + 4096 image tokens,
q/k/v ~N(0,1), per-head QK-RMSNorm with weight 1 and the v1 3D RoPE on the
(1, 64, 64) grid, seed 2) plus ragged lengths (49, 257, 777).
"""
import pytest
import torch

from oracle import sage_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _needs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not sage_ref.available():
        pytest.skip("the reference SageAttention is not built (oracle/build_sage_ref.py)")


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm())).item()


def _rms_rope(x, freqs):
    """Diffusers RMSNorm (weight 1, eps 1e-6; two roundings) then
    apply_rotary_emb_qwen(use_real=False) in torch on the GPU."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    xc = torch.view_as_complex(y.float().reshape(*y.shape[:-1], -1, 2))
    return torch.view_as_real(xc * freqs[None, :, None, :]).flatten(3).to(torch.bfloat16)


def config3_inputs(b=2, h=24, lt=256, grid=64, seed=2):
    from qwen_image_accel_b200.mmdit import rope_tables
    g = torch.Generator(device=DEV).manual_seed(seed)
    s = lt + grid * grid
    q, k, v = (torch.randn(b, s, h, 128, device=DEV, dtype=torch.bfloat16, generator=g) for _ in range(3))
    img, txt = rope_tables(1, grid, grid, lt)
    freqs = torch.cat([txt, img]).to(DEV)
    return _rms_rope(q, freqs), _rms_rope(k, freqs), v


def ragged_inputs(b, s, h, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q, k, v = (torch.randn(b, s, h, 128, device=DEV, dtype=torch.bfloat16, generator=g) for _ in range(3))
    return q, k + 0.25, v  # a non-zero K mean exercises the smoothing


CASES = [("config3", None), ("s49", (1, 49, 2)), ("s257", (2, 257, 3)), ("s777", (1, 777, 2))]


def _inputs(name, spec):
    return config3_inputs() if spec is None else ragged_inputs(*spec, seed=len(name))


def _ours(q, k, v):
    from qwen_image_accel_b200.optimizations.sage_attention import sage_quantize
    b, s, h, _ = q.shape
    ws = sage_quantize(q, k, v)
    nhd = lambda t: t.view(b, h, -1, 128)[:, :, :s].permute(0, 2, 1, 3)  # noqa: E731
    return {"q8": nhd(ws["q8"]), "k8": nhd(ws["k8"]), "v8": nhd(ws["v8"].view(torch.uint8)),
            "q_scale": ws["q_scale"].view(b, h, -1), "k_scale": ws["k_scale"].view(b, h, -1),
            "v_scale": ws["v_scale"].view(b, h, 128), "k_mean": ws["k_mean"].view(b, h, 128)}


@pytest.mark.parametrize("name,spec", CASES, ids=[c[0] for c in CASES])
def test_quantizers_vs_sage(name, spec):
    q, k, v = _inputs(name, spec)
    b, s, h, _ = q.shape
    mine = _ours(q, k, v)

    # Q: codes and scales bit-exact
    q8, qs, _, _ = sage_ref.quantize_qk(q, k)
    assert torch.equal(mine["q8"], q8), f"Q codes: {(mine['q8'] != q8).sum().item()} differ"
    assert torch.equal(mine["q_scale"][..., :qs.shape[-1]], qs), "Q scales differ"

    # the smoothing mean: within 1 bf16 ulp of torch's k.mean, rarely different
    km_torch = sage_ref.k_mean(k).squeeze(1)                      # [B, H, d] bf16
    km_mine = mine["k_mean"]
    ulps = (km_mine.view(torch.int16).int() - km_torch.view(torch.int16).int()).abs()
    n_diff = int((ulps != 0).sum())
    assert int(ulps.max()) <= 1, f"K mean: max {int(ulps.max())} ulp from torch's k.mean"
    assert n_diff * 500 <= km_torch.numel(), f"K mean: {n_diff} of {km_torch.numel()} elements differ"

    # K: bit-exact given the same mean
    _, _, k8_same, ks_same = sage_ref.quantize_qk(q, k, km=km_mine[:, None])
    nk = ks_same.shape[-1]
    assert torch.equal(mine["k8"], k8_same), f"K codes (same mean): {(mine['k8'] != k8_same).sum().item()} differ"
    assert torch.equal(mine["k_scale"][..., :nk], ks_same), "K scales (same mean) differ"
    # against Sage's own mean: differences only where the mean differs, by <= 1
    _, _, k8_ref, _ = sage_ref.quantize_qk(q, k)
    dk = (mine["k8"].int() - k8_ref.int()).abs()
    assert int(dk.max()) <= 1
    chan_diff = (ulps != 0)                                        # [B, H, d]
    assert not bool((dk.amax(dim=1) > 0)[~chan_diff].any()), "a K code differs in a channel whose mean agrees"

    # V: codes (Sage's 16-key permutation undone) and scales bit-exact
    v8_ref, vs_ref = sage_ref.quantize_v(v)
    v8_seq = sage_ref.unpermute_v(v8_ref)[:, :s]
    assert torch.equal(mine["v8"], v8_seq), f"V codes: {(mine['v8'] != v8_seq).sum().item()} differ"
    assert torch.equal(mine["v_scale"], vs_ref), "V scales differ"


@pytest.mark.parametrize("name,spec", CASES, ids=[c[0] for c in CASES])
def test_attention_vs_sage(name, spec):
    from qwen_image_accel_b200 import _lib
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention
    q, k, v = _inputs(name, spec)
    ref = sage_ref.attention(q, k, v)
    out = sage_attention(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.isfinite(out).all() and torch.isfinite(ref).all()
    c = cosine(out, ref)
    assert c >= 0.999, f"cosine {c} against the reference SageAttention"
    err = (out.float() - ref.float()).abs().max().item()
    assert err <= 0.05 * ref.float().abs().max().item(), f"max abs diff {err}"
