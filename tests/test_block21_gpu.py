"""The Qwen-Image 2.1 single-stream block on the sm_100a kernels
(qwen21.Block21) against the Diffusers QwenImage21TransformerBlock golden
(tests/golden/block21_tiny.npz: dim 512, 4 x 128 heads, a condition-image
edit sequence of 138 tokens with a 74-token prefix): the prefill with the
prefix K/V extracted, and a cached decode of new target tokens, per profile.

Gates (printed per profile): the stored prefix K/V and both outputs against
the bf16 eager CPU reference, by PSNR and cosine -- tighter for the bf16
profiles, looser where the MXFP8 linears and the INT8/FP8 attention
quantize. The cached decode is also run on the golden's own cache, which
isolates it from the prefill's differences.
"""
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


def build(profile, sage_prefill=False):
    from qwen_image_accel_b200.mmdit import init_parameter
    from qwen_image_accel_b200.qwen21 import Block21, Block21Config, block21_parameter_shapes
    g = np.load(GOLD / "block21_tiny.npz")
    dim, heads = g["dims"].tolist()
    cfg = Block21Config(dim=dim, heads=heads)
    shapes = block21_parameter_shapes(cfg)
    assert sorted(shapes) == sorted(g["keys"].tolist())
    blk = Block21(lambda n: init_parameter(n, shapes[n], seed=11), cfg, device="cuda", profile=profile,
                  sage_prefill=sage_prefill)
    return blk, g


# profile, sage_prefill, min PSNR (dB), min cosine
# (measured on B200: bf16 profiles 75-119 dB, MXFP8 profiles 47-67 dB, every cosine >= 0.99928)
CASES = [("fused", False, 60.0, 0.99999), ("fused_sage", False, 55.0, 0.99999), ("fused_sage", True, 55.0, 0.9999),
         ("mxfp8", False, 40.0, 0.999), ("mxfp8_sage", False, 40.0, 0.999), ("mxfp8_sage", True, 40.0, 0.999)]


@pytest.mark.parametrize("profile,sage_prefill,min_psnr,min_cos", CASES)
def test_prefill_extract_then_cached_decode(profile, sage_prefill, min_psnr, min_cos):
    from qwen_image_accel_b200.qwen21 import KVLayerCache, modulation_values
    blk, g = build(profile, sage_prefill)
    h, mod, ht = (t_bf16(g[n]).cuda() for n in ("h", "modulation", "h_target"))
    freqs = torch.view_as_complex(torch.from_numpy(g["rope"]).contiguous()).cuda()
    ids = torch.from_numpy(g["image_ids"]).cuda()
    p = int(g["prefix_len"])
    cache = KVLayerCache()
    out_pre = blk.forward_prefill(h, mod, freqs, ids, p, layer_cache=cache).float().cpu()
    ck, cv = (t.float().cpu() for t in cache.get())
    ref_pre, ref_k, ref_v = (t_bf16(g[n]).float() for n in ("out_prefill", "cached_k", "cached_v"))
    vals = modulation_values(mod)
    out_dec = blk.forward_cached(ht, vals, freqs[p:], cache).float().cpu()
    gold_cache = KVLayerCache()
    gold_cache.store(t_bf16(g["cached_k"]).cuda(), t_bf16(g["cached_v"]).cuda())
    out_dec_gold = blk.forward_cached(ht, vals, freqs[p:], gold_cache).float().cpu()
    ref_dec = t_bf16(g["out_cached"]).float()
    figures = {"prefill": (out_pre, ref_pre), "cached_k": (ck, ref_k), "cached_v": (cv, ref_v),
               "decode": (out_dec, ref_dec), "decode_on_golden_cache": (out_dec_gold, ref_dec)}
    report = {k: (round(psnr(a, b), 2), round(cosine(a, b), 6)) for k, (a, b) in figures.items()}
    print(profile, "sage_prefill" if sage_prefill else "sdpa_prefill", report)
    for name, (a, _) in figures.items():
        assert torch.isfinite(a).all(), name
    for name, (pv, cv_) in report.items():
        assert pv >= min_psnr and cv_ >= min_cos, (name, pv, cv_)


def test_bf16_decode_on_golden_cache_is_tight():
    """bf16 profile, decode on the reference's own cache: only LN order,
    GEMM accumulation order and the SDPA kernel differ from the eager CPU
    block."""
    from qwen_image_accel_b200.qwen21 import KVLayerCache, modulation_values
    blk, g = build("fused")
    mod, ht = t_bf16(g["modulation"]).cuda(), t_bf16(g["h_target"]).cuda()
    freqs = torch.view_as_complex(torch.from_numpy(g["rope"]).contiguous()).cuda()
    p = int(g["prefix_len"])
    cache = KVLayerCache()
    cache.store(t_bf16(g["cached_k"]).cuda(), t_bf16(g["cached_v"]).cuda())
    out = blk.forward_cached(ht, modulation_values(mod), freqs[p:], cache).float().cpu()
    ref = t_bf16(g["out_cached"]).float()
    assert psnr(out, ref) >= 45.0 and cosine(out, ref) >= 0.99999


def test_fused_decode_equals_reference_op_composition():
    """MXFP8 + Sage decode: the fused block (stacked Q|K|V GEMM, segment
    norm/RoPE into the joint buffers, MXFP8 attention output, gate-residual
    epilogues, grouped gate/value GEMMs) is byte-identical to the reference's
    op sequence on the same kernels (quantized_decode.py:31-137: three
    projections of one activation, prepare_attention_inputs, sage_decode,
    to_out, residual, _mx_mlp_forward, residual)."""
    import torch.nn as nn
    from qwen_image_accel_b200.kernels.attention import prepare_attention_inputs
    from qwen_image_accel_b200.kernels.elementwise import residual
    from qwen_image_accel_b200.kernels.epilogue import layer_norm_scale_quantize, swiglu_quantize
    from qwen_image_accel_b200.mmdit import init_parameter
    from qwen_image_accel_b200.optimizations.mxfp8 import MXFP8Linear
    from qwen_image_accel_b200.optimizations.sage_attention import sage_attention
    from qwen_image_accel_b200.qwen21 import KVLayerCache, block21_parameter_shapes, Block21Config, modulation_values
    blk, g = build("mxfp8_sage")
    dim, heads = g["dims"].tolist()
    shapes = block21_parameter_shapes(Block21Config(dim=dim, heads=heads))

    def mx(name):
        w = init_parameter(name, shapes[name], seed=11).cuda()
        lin = nn.Linear(w.shape[1], w.shape[0], bias=False, device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(w)
        return MXFP8Linear(lin)

    to_q, to_k, to_v = (mx(f"attn.to_{n}.weight") for n in "qkv")
    mod, ht = t_bf16(g["modulation"]).cuda(), t_bf16(g["h_target"]).cuda()
    freqs = torch.view_as_complex(torch.from_numpy(g["rope"]).contiguous()).cuda()
    p = int(g["prefix_len"])
    ck, cv = t_bf16(g["cached_k"]).cuda(), t_bf16(g["cached_v"]).cuda()
    s1, g1, s2, g2 = vals = modulation_values(mod)
    b, st, d = ht.shape
    a = layer_norm_scale_quantize(ht, s1, blk.norm)
    q, k, v = (lin.matmul(a).view(b, st, heads, 128) for lin in (to_q, to_k, to_v))
    q, k, v = prepare_attention_inputs(q, k, v, blk.norm_q, blk.norm_k, freqs[p:].contiguous(), ck, cv)
    h1 = residual(ht, blk.to_out(sage_attention(q, k, v).flatten(2, 3).contiguous()), g1)
    a2 = layer_norm_scale_quantize(h1, s2, blk.norm)
    act = swiglu_quantize(blk.gate_layer.matmul(a2), blk.proj.matmul(a2))
    want = residual(h1, blk.out.matmul(act).view(b, st, d), g2)
    cache = KVLayerCache()
    cache.store(ck, cv)
    got = blk.forward_cached(ht, vals, freqs[p:].contiguous(), cache)
    assert torch.equal(got, want)


@pytest.mark.parametrize("sage_prefill", [False, True])
def test_batch_of_two_equals_single_samples(sage_prefill):
    """B = 2 (the golden sample twice, one shared modulation row set) gives
    each sample the B = 1 result bit for bit, in the prefill (per-sample
    modulation rows, extracted K/V) and in the cached decode (joint K/V
    buffers, gate-residual epilogue rows per sample)."""
    from qwen_image_accel_b200.qwen21 import KVLayerCache, modulation_values
    blk, g = build("mxfp8_sage", sage_prefill)
    h, mod, ht = (t_bf16(g[n]).cuda() for n in ("h", "modulation", "h_target"))
    freqs = torch.view_as_complex(torch.from_numpy(g["rope"]).contiguous()).cuda()
    ids = torch.from_numpy(g["image_ids"]).cuda()
    p = int(g["prefix_len"])
    mod2 = torch.cat([mod[:1], mod[:1], mod[1:]])             # two sampled rows + the t = 0 row
    c1, c2 = KVLayerCache(), KVLayerCache()
    one = blk.forward_prefill(h, mod, freqs, ids, p, layer_cache=c1)
    two = blk.forward_prefill(torch.cat([h, h]), mod2, freqs, ids, p, layer_cache=c2)
    assert torch.equal(two[0], one[0]) and torch.equal(two[1], one[0])
    assert torch.equal(c2.k[1], c1.k[0]) and torch.equal(c2.v[0], c1.v[0])
    d1 = blk.forward_cached(ht, modulation_values(mod), freqs[p:].contiguous(), c1)
    d2 = blk.forward_cached(torch.cat([ht, ht]), modulation_values(mod2), freqs[p:].contiguous(), c2)
    assert torch.equal(d2[0], d1[0]) and torch.equal(d2[1], d1[0])
