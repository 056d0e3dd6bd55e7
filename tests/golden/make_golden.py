"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs only where the reference checkout is mounted (it is read, never
modified). Sources of truth, per fixture:

* mxfp8_quantize.npz -- E8M0 scales from the reference's own Triton kernel
  `_mx_quantize_kernel` (src/qwen_image_accel/kernels/mxfp8.py:31) run by the
  Triton interpreter on the CPU; codes from the reference's known-answer rule
  (tests/gpu/check_mxfp8.py:41-51): x * 2^(127-e) cast with torch's
  float8_e4m3fn. (The interpreter's own fp8/bf16 casts truncate, so its codes
  are not used.) Shapes and the outlier pattern follow check_mxfp8.py:59-62.
* residual.npz -- eager `h + gate * x` in bf16, the oracle of the reference's
  residual check (tests/gpu/check_fused.py:197-198).
* ln_mod.npz -- eager bf16 `LayerNorm(x) * (1 + s) + shift` (CPU order; the
  CUDA-order pin runs on the GPU against torch's CUDA LayerNorm).
* rope_rms.npz -- Diffusers RMSNorm and apply_rotary_emb_qwen(use_real=False)
  from the pinned wheel (the oracle of tests/gpu/check_attention_ops.py:264-267),
  with freqs from QwenEmbedRope for a (1, 4, 4) grid and 16 text tokens.
* activations.npz -- eager F.silu(g) * v and F.gelu(x, approximate="tanh").
* block_causal.npz -- the Qwen-Image 2.1 prefill mask (token metadata,
  prefix segments and the flex mask_mod evaluated densely, with a key-padding
  mask) from WHL:diffusers/models/transformers/transformer_qwenimage21.py.
* block21_tiny.npz -- one Qwen-Image 2.1 single-stream block (Diffusers
  QwenImage21TransformerBlock, tiny dims, seeded weights): prefill with the
  prefix K/V extracted, then a cached decode of new target tokens.
* model21_tiny.npz -- the whole Qwen-Image 2.1 transformer (Diffusers
  QwenImage21Transformer2DModel, 2 blocks, tiny dims, seeded weights):
  prefill with KV extract, then one cached step.
* mmdit_tiny.npz -- the Diffusers QwenImageTransformer2DModel (v1 dual-stream
  MMDiT, WHL:diffusers/models/transformers/transformer_qwenimage.py) at a tiny
  size (2 blocks, 4x128 heads, text dim 512) in bf16 on the CPU, weights from
  the package's seeded recipe (mmdit.init_parameter, torch CPU generator),
  seeded inputs; plus its RoPE tables and timestep embedding input.

Usage: python tests/golden/make_golden.py --reference /path/to/checkout  (or QIA_REFERENCE=...)
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
import types
import zipfile
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _import_diffusers(reference: Path):
    whl = next((reference / "third_party" / "wheels").glob("diffusers-*.whl"))
    dest = Path(tempfile.mkdtemp(prefix="qia_golden_whl_"))
    with zipfile.ZipFile(whl) as z:
        z.extractall(dest)
    sys.path.insert(0, str(dest))
    import huggingface_hub
    import huggingface_hub.errors
    import huggingface_hub.utils
    # attributes the pinned wheel imports but the installed hub release lacks
    for mod, name, val in [(huggingface_hub, "resolve_revision", lambda *a, **k: None),
                           (huggingface_hub.errors, "RevisionResolutionError",
                            type("RevisionResolutionError", (Exception,), {})),
                           (huggingface_hub.utils, "httpx", types.SimpleNamespace())]:
        if not hasattr(mod, name):
            setattr(mod, name, val)


def make_mxfp8(reference: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(reference / "src"))
    import torch
    from qwen_image_accel.kernels import mxfp8
    torch.manual_seed(0)
    cases = {}
    for m, k in [(1, 128), (77, 256), (130, 256), (200, 384)]:
        x = torch.randn(m, k, dtype=torch.bfloat16)
        x[:, ::64] *= 40
        if m > 100:
            x[m // 3] *= 1e-3
        a = mxfp8.quantize(x)
        padded = a.values.shape[0]
        scales = a.scales.view(torch.uint8)
        # unswizzle the kernel's exponents back to [padded, k/32]
        e = scales.view(padded // 128, k // 128, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(padded, k // 32)
        xp = torch.zeros(padded, k, dtype=torch.bfloat16)
        xp[:m] = x
        codes = (xp.float().view(padded, k // 32, 32) * torch.exp2(127 - e.float())[..., None]
                 ).to(torch.float8_e4m3fn).view(torch.uint8).view(padded, k)
        cases[f"x_{m}_{k}"] = _bits(x)
        cases[f"codes_{m}_{k}"] = codes.numpy()
        cases[f"scales_{m}_{k}"] = scales.numpy().copy()
    np.savez_compressed(OUT / "mxfp8_quantize.npz", **cases)


def make_eager(reference: Path):
    import torch
    import torch.nn.functional as F
    _import_diffusers(reference)
    from diffusers.models.normalization import RMSNorm
    from diffusers.models.transformers.transformer_qwenimage import QwenEmbedRope, apply_rotary_emb_qwen

    torch.manual_seed(91)
    res = {}
    for b, s, d in [(1, 49, 256), (2, 9, 512)]:
        h = torch.randn(b, s, d, dtype=torch.bfloat16)
        x = torch.randn_like(h)
        g = torch.randn(b, 1, d, dtype=torch.bfloat16).tanh()
        res[f"h_{b}_{s}_{d}"], res[f"x_{b}_{s}_{d}"], res[f"g_{b}_{s}_{d}"] = _bits(h), _bits(x), _bits(g)
        res[f"out_{b}_{s}_{d}"] = _bits(h + g * x)
    np.savez_compressed(OUT / "residual.npz", **res)

    torch.manual_seed(717)
    ln = {}
    for b, s, d in [(1, 7, 512), (2, 3, 1536), (1, 2, 3072)]:
        x = torch.randn(b, s, d, dtype=torch.bfloat16) * 3
        sc = (1 + 0.1 * torch.randn(b, 1, d)).to(torch.bfloat16)
        sh = (0.1 * torch.randn(b, 1, d)).to(torch.bfloat16)
        norm = torch.nn.LayerNorm(d, elementwise_affine=False, eps=1e-6)
        key = f"{b}_{s}_{d}"
        ln[f"x_{key}"], ln[f"scale_{key}"], ln[f"shift_{key}"] = _bits(x), _bits(sc), _bits(sh)
        ln[f"out_{key}"] = _bits(norm(x) * sc + sh)
        ln[f"noshift_{key}"] = _bits(norm(x) * sc)
    np.savez_compressed(OUT / "ln_mod.npz", **ln)

    torch.manual_seed(721)
    rr = {}
    rope = QwenEmbedRope(theta=10000, axes_dim=[16, 56, 56], scale_rope=True)
    img_freqs, txt_freqs = rope([(1, 4, 4)], max_txt_seq_len=16, device=torch.device("cpu"))
    rr["img_freqs"] = torch.view_as_real(img_freqs).numpy().copy()
    rr["txt_freqs"] = torch.view_as_real(txt_freqs).numpy().copy()
    nq = RMSNorm(128, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        nq.weight.copy_(torch.randn(128))
    q = torch.randn(2, 16, 3, 128, dtype=torch.bfloat16) * 2
    with torch.no_grad():
        normed = nq(q)
        rot = apply_rotary_emb_qwen(normed, img_freqs, use_real=False)
    rr["q"], rr["w"], rr["normed"], rr["rotated"] = _bits(q), _bits(nq.weight.data), _bits(normed), _bits(rot)
    np.savez_compressed(OUT / "rope_rms.npz", **rr)

    torch.manual_seed(5)
    act = {}
    g = torch.randn(32, 128, dtype=torch.bfloat16) * 3
    v = torch.randn(32, 128, dtype=torch.bfloat16)
    act["g"], act["v"], act["swiglu"] = _bits(g), _bits(v), _bits(F.silu(g) * v)
    x = torch.randn(32, 128, dtype=torch.bfloat16) * 4
    act["x"], act["gelu"] = _bits(x), _bits(F.gelu(x, approximate="tanh"))
    np.savez_compressed(OUT / "activations.npz", **act)


def make_mmdit(reference: Path):
    import torch
    _import_diffusers(reference)
    from diffusers.models.transformers.transformer_qwenimage import QwenImageTransformer2DModel
    sys.path.insert(0, str(OUT.parents[1] / "qwen-image-2.1-accel_b200"))
    from qwen_image_accel_b200.mmdit import MMDiTConfig, init_parameter, parameter_shapes, rope_tables

    cfg = MMDiTConfig(num_layers=2, num_attention_heads=4, joint_attention_dim=512)
    model = QwenImageTransformer2DModel(patch_size=2, in_channels=64, out_channels=16, num_layers=2,
                                        attention_head_dim=128, num_attention_heads=4, joint_attention_dim=512,
                                        axes_dims_rope=(16, 56, 56)).to(torch.bfloat16)
    shapes = parameter_shapes(cfg)
    sd = model.state_dict()
    assert set(sd) == set(shapes), sorted(set(sd) ^ set(shapes))
    model.load_state_dict({n: init_parameter(n, shapes[n], seed=7) for n in sd})
    model.eval()
    g = torch.Generator().manual_seed(42)
    f, h, w, lt = 1, 12, 16, 40
    x = torch.randn(2, f * h * w, 64, generator=g).to(torch.bfloat16)
    enc = torch.randn(2, lt, 512, generator=g).to(torch.bfloat16)
    t = torch.tensor([0.7, 0.7]).to(torch.bfloat16)
    with torch.no_grad():
        out = model(hidden_states=x, encoder_hidden_states=enc, timestep=t, img_shapes=[(f, h, w)] * 2,
                    return_dict=False)[0]
        img_f, txt_f = model.pos_embed([(f, h, w)], max_txt_seq_len=lt, device=torch.device("cpu"))
    mine_img, mine_txt = rope_tables(f, h, w, lt)
    assert torch.equal(mine_img, img_f) and torch.equal(mine_txt, txt_f)
    np.savez_compressed(OUT / "mmdit_tiny.npz", x=_bits(x), enc=_bits(enc), out=_bits(out),
                        img_freqs=torch.view_as_real(img_f).numpy().copy(),
                        txt_freqs=torch.view_as_real(txt_f).numpy().copy(),
                        shape=np.array([f, h, w, lt]), timestep=np.float32(0.7),
                        keys=np.array(sorted(sd)))


def make_block_causal(reference: Path):
    """The 2.1 prefill mask from the pinned wheel: token metadata
    (QwenImage21Transformer2DModel.build_token_metadata), the prefix segments
    the default processor iterates (_qwenimage21_prefix_segments) and the
    dense mask of the flex BlockMask's mask_mod
    (build_qwenimage21_block_causal_mask), for a few sequence layouts."""
    import torch
    _import_diffusers(reference)
    from diffusers.models.transformers import transformer_qwenimage21 as t21

    # (runs of (kind, length) in sequence order, image shapes condition-first)
    layouts = {
        "t2i": ([("t", 7), ("i", 8)], [(1, 2, 4)]),
        "edit": ([("t", 5), ("i", 6), ("t", 3), ("i", 8)], [(1, 2, 3), (1, 2, 4)]),
        "adjacent": ([("t", 4), ("i", 4), ("i", 6), ("t", 2), ("i", 12)], [(1, 2, 2), (1, 2, 3), (1, 3, 4)]),
        "long": ([("t", 37), ("i", 64), ("t", 11), ("i", 48), ("t", 5), ("i", 96)], [(1, 8, 8), (1, 6, 8), (1, 8, 12)]),
    }
    cases = {}
    for name, (runs, shapes) in layouts.items():
        pad = torch.cat([torch.full((n,), kind == "i") for kind, n in runs])
        image_ids, target = t21.QwenImage21Transformer2DModel.build_token_metadata(pad, shapes)
        s = pad.shape[0]
        prefix_len = int((~target).sum())
        segments = t21._qwenimage21_prefix_segments(image_ids, prefix_len)
        g = torch.Generator().manual_seed(len(name))
        key_valid = torch.ones(2, s, dtype=torch.bool)
        text_pos = (~pad).nonzero(as_tuple=True)[0]
        drop = text_pos[torch.randperm(text_pos.numel(), generator=g)[: max(1, text_pos.numel() // 4)]]
        key_valid[1, drop] = False
        key_valid[1, 0] = True
        bm = t21.build_qwenimage21_block_causal_mask(image_ids, key_valid, 2, torch.device("cpu"))
        qi = torch.arange(s)[:, None]
        ki = torch.arange(s)[None, :]
        dense = torch.stack([bm.mask_mod(torch.tensor(b), torch.tensor(0), qi, ki) for b in range(2)])
        cases[f"image_ids_{name}"] = image_ids.numpy().astype(np.int64)
        cases[f"target_{name}"] = target.numpy()
        cases[f"segments_{name}"] = np.array([(a, b, int(t)) for a, b, t in segments], np.int64).reshape(-1, 3)
        cases[f"key_valid_{name}"] = key_valid.numpy()
        cases[f"mask_{name}"] = dense.numpy()
    np.savez_compressed(OUT / "block_causal.npz", **cases)


BLOCK21_RUNS = [("t", 20), ("i", 48), ("t", 6), ("i", 64)]      # text, condition image, text, target
BLOCK21_SHAPES = [(1, 6, 8), (1, 8, 8)]


def make_block21(reference: Path):
    """One Diffusers QwenImage21TransformerBlock (dim 512, 4 x 128 heads, SwiGLU
    1536) in bf16 on the CPU, weights from the package's seeded recipe
    (mmdit.init_parameter, seed 11): the prefill of a condition-image edit
    sequence with the prefix K/V extracted into a QwenImage21KVLayerCache
    (kv_cache_mode="extract", the default per-segment processor), then one
    cached decode of new target tokens (kv_cache_mode="cached")."""
    import torch
    _import_diffusers(reference)
    from diffusers.models.transformers import transformer_qwenimage21 as t21
    sys.path.insert(0, str(OUT.parents[1] / "qwen-image-2.1-accel_b200"))
    from qwen_image_accel_b200.mmdit import init_parameter

    dim, heads = 512, 4
    block = t21.QwenImage21TransformerBlock(dim, heads, 128).to(torch.bfloat16)
    sd = block.state_dict()
    block.load_state_dict({n: init_parameter(n, tuple(t.shape), seed=11) for n, t in sd.items()})
    block.eval()
    pad = torch.cat([torch.full((n,), kind == "i") for kind, n in BLOCK21_RUNS])
    image_ids, target = t21.QwenImage21Transformer2DModel.build_token_metadata(pad, BLOCK21_SHAPES)
    prefix_len = int((~target).sum())
    segments = t21._qwenimage21_prefix_segments(image_ids, prefix_len)
    rope = t21.QwenImage21Rope(theta=10000, axes_dim=[16, 56, 56])(BLOCK21_SHAPES, pad, torch.device("cpu"))
    g = torch.Generator().manual_seed(21)
    s = pad.shape[0]
    h = torch.randn(1, s, dim, generator=g).to(torch.bfloat16)
    modulation = (0.5 * torch.randn(2, 4 * dim, generator=g)).to(torch.bfloat16)   # [real row, t = 0 row]
    h_target = torch.randn(1, s - prefix_len, dim, generator=g).to(torch.bfloat16)
    cache = t21.QwenImage21KVLayerCache()
    with torch.no_grad():
        out_prefill = block(hidden_states=h, modulation=modulation, rotary_emb=rope, attention_mask=None,
                            target_token_mask=target, layer_cache=cache, kv_cache_mode="extract",
                            cache_write_slice=slice(0, prefix_len), segments=segments, key_valid=None)
        cached_k, cached_v = cache.get()
        out_cached = block(hidden_states=h_target, modulation=modulation, rotary_emb=rope[prefix_len:],
                           attention_mask=None, target_token_mask=target[prefix_len:], layer_cache=cache,
                           kv_cache_mode="cached", cache_write_slice=None, segments=None, key_valid=None)
    np.savez_compressed(OUT / "block21_tiny.npz", h=_bits(h), modulation=_bits(modulation),
                        h_target=_bits(h_target), out_prefill=_bits(out_prefill), out_cached=_bits(out_cached),
                        cached_k=_bits(cached_k), cached_v=_bits(cached_v), image_ids=image_ids.numpy(),
                        target=target.numpy(), rope=torch.view_as_real(rope).numpy().copy(),
                        prefix_len=np.int64(prefix_len), dims=np.array([dim, heads]),
                        keys=np.array(sorted(sd)))


def make_model21(reference: Path):
    """The whole Diffusers QwenImage21Transformer2DModel at a tiny size (2
    blocks, 4 x 128 heads, text dim 256) in bf16 on the CPU, weights from the
    package's seeded recipe (seed 13): a condition-image edit in the
    vision-language slot layout (text 10, condition image (1, 4, 4) as 4
    slots, text 3, target (1, 4, 6) as 6 slots), prefill with kv_cache_mode
    "extract" at t = 0.8, then a cached step at t = 0.6 with new target
    latents."""
    import torch
    _import_diffusers(reference)
    from diffusers.models.transformers import transformer_qwenimage21 as t21
    sys.path.insert(0, str(OUT.parents[1] / "qwen-image-2.1-accel_b200"))
    from qwen_image_accel_b200.mmdit import init_parameter

    model = t21.QwenImage21Transformer2DModel(num_layers=2, num_attention_heads=4, context_in_dim=256).to(torch.bfloat16)
    sd = model.state_dict()
    model.load_state_dict({n: init_parameter(n, tuple(t.shape), seed=13) for n, t in sd.items()})
    model.eval()
    shapes = [(1, 4, 4), (1, 4, 6)]
    img_mask = torch.tensor([[False] * 10 + [True] * 4 + [False] * 3 + [True] * 6])
    g = torch.Generator().manual_seed(31)
    enc = torch.randn(1, img_mask.shape[1] - 6, 256, generator=g).to(torch.bfloat16)
    lat = torch.randn(1, 16 + 24, 64, generator=g).to(torch.bfloat16)
    lat2 = lat.clone()
    lat2[:, 16:] = torch.randn(1, 24, 64, generator=g).to(torch.bfloat16)
    cache = t21.QwenImage21KVCache(2)
    with torch.no_grad():
        out_prefill = model(hidden_states=lat, encoder_hidden_states=enc, timestep=torch.tensor([0.8]),
                            img_shapes=[shapes], img_mask=img_mask, kv_cache=cache, kv_cache_mode="extract",
                            return_dict=False)[0]
        out_cached = model(hidden_states=lat2, encoder_hidden_states=enc, timestep=torch.tensor([0.6]),
                           img_shapes=[shapes], img_mask=img_mask, kv_cache=cache, kv_cache_mode="cached",
                           return_dict=False)[0]
    np.savez_compressed(OUT / "model21_tiny.npz", lat=_bits(lat), lat2=_bits(lat2), enc=_bits(enc),
                        img_mask=img_mask.numpy(), shapes=np.array(shapes), out_prefill=_bits(out_prefill),
                        out_cached=_bits(out_cached), cached_k0=_bits(cache.get_layer(0).k),
                        keys=np.array(sorted(sd)), t=np.array([0.8, 0.6], np.float32))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QIA_REFERENCE"),
                    help="reference checkout (read only); or set QIA_REFERENCE")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or QIA_REFERENCE) is required")
    ref = Path(args.reference)
    make_mxfp8(ref)   # first: the interpreter flag must precede the first triton import
    make_eager(ref)
    make_mmdit(ref)
    make_block_causal(ref)
    make_block21(ref)
    make_model21(ref)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))
