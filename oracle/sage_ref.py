"""The reference's SageAttention, built from its pinned sources, as a checker --
TEST INFRASTRUCTURE, never the product.

`oracle/build_sage_ref.py` compiles the SageAttention 2.2.0 extension modules
(`sage_ref_fused`, `sage_ref_qattn`) into oracle/_ref/sage/. This module loads
them and restates, step for step, the Python around them that the reference's
`qw21::sage_decode` runs (src/qwen_image_accel/optimizations/sage_attention.py:
19-25 -> SAGE:sageattention/core.py:636-828 with tensor_layout="NHD",
is_causal=False, qk_quant_gran="per_warp", pv_accum_dtype="fp32+fp32",
smooth_k=True, smooth_v=False):

* K smoothing mean: `k.mean(dim=1, keepdim=True)` in torch (core.py:773);
* Q INT8 per 32-row warp block, K INT8 per 64-row block of k - mean
  (SAGE:sageattention/quant.py:105-179 -> fused.cu quant_per_warp_int8_cuda,
  quant_per_block_int8_fuse_sub_mean_cuda);
* V FP8 E4M3 per channel, scale_max 448, transposed/padded/permuted to
  [B, d, H, S_pad64] (quant.py:224-292 -> transpose_pad_permute_cuda,
  scale_fuse_quant_cuda);
* the attention kernel qk_int8_sv_f8_accum_f32_fuse_v_scale_attn_inst_buf
  (core.py:816-817), sm_scale = d^-0.5.

Only tests/ and bench.py's checker legs import this module.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref" / "sage"

_mods: dict = {}


def available() -> bool:
    return all((REF / n / f"{n}.so").exists() for n in ("sage_ref_fused", "sage_ref_qattn"))


def _load(name: str):
    if name not in _mods:
        import torch  # noqa: F401  (the extension links against torch's libraries)
        path = REF / name / f"{name}.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with oracle/build_sage_ref.py")
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        _mods[name] = mod
    return _mods[name]


def k_mean(k):
    """core.py:773 -- the smoothing mean of K over the sequence, NHD [B, S, H, d] -> [B, 1, H, d]."""
    return k.mean(dim=1, keepdim=True)


def quantize_qk(q, k, km=None):
    """quant.py:105-179 (per_warp_int8, NHD, BLKQ=128, WARPQ=32, BLKK=64):
    (q_int8 [B,S,H,d], q_scale [B,H,ceil(S/128)*4], k_int8, k_scale [B,H,ceil(Skv/64)]).
    km: the [B, 1, H, d] mean (k_mean(k) when None)."""
    import torch
    fused = _load("sage_ref_fused")
    if km is None:
        km = k_mean(k)
    b, sq, h, _ = q.shape
    skv, hk = k.shape[1], k.shape[2]
    q8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    k8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    qs = torch.empty((b, h, (sq + 127) // 128 * 4), device=q.device, dtype=torch.float32)
    ks = torch.empty((b, hk, (skv + 63) // 64), device=q.device, dtype=torch.float32)
    fused.quant_per_warp_int8_cuda(q, q8, qs, 128, 32, 0)
    fused.quant_per_block_int8_fuse_sub_mean_cuda(k, km.squeeze(1), k8, ks, 64, 0)
    return q8, qs, k8, ks


def quantize_v(v, scale_max: float = 448.0):
    """quant.py:224-292 (per_channel_fp8, NHD, smooth_v=False): (v_fp8
    [B, d, H, S_pad64] in Sage's permuted key order, v_scale [B, H, d])."""
    import torch
    fused = _load("sage_ref_fused")
    b, skv, h, d = v.shape
    pad = (skv + 63) // 64 * 64
    vt = torch.empty((b, d, h, pad), dtype=v.dtype, device=v.device)
    fused.transpose_pad_permute_cuda(v, vt, 0)
    v8 = torch.empty(vt.shape, dtype=torch.float8_e4m3fn, device=v.device)
    vs = torch.empty((b, h, d), dtype=torch.float32, device=v.device)
    fused.scale_fuse_quant_cuda(vt, v8, vs, skv, scale_max, 0)
    return v8, vs


# Sage's V layout permutes keys inside every 16-key group (quant.py:230-233).
PERM16 = (0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15)


def unpermute_v(v8):
    """[B, d, H, S_pad] in Sage's key order -> [B, S_pad, H, d] in sequence order."""
    import torch
    b, d, h, s = v8.shape
    inv = [0] * 16
    for i, p in enumerate(PERM16):
        inv[p] = i
    idx = torch.tensor(inv, device=v8.device)
    g = v8.view(torch.uint8).view(b, d, h, s // 16, 16)[..., idx]
    return g.reshape(b, d, h, s).permute(0, 3, 2, 1).contiguous()


def attention(q, k, v, sm_scale: float | None = None):
    """sageattn_qk_int8_pv_fp8_cuda(q, k, v, "NHD", per_warp, fp32+fp32),
    q/k/v bf16 NHD [B, S, H, 128] -> bf16 NHD (core.py:725-828)."""
    import torch
    qattn = _load("sage_ref_qattn")
    d = q.shape[-1]
    if d != 128:
        raise ValueError("the checker covers head_dim 128 only")
    if sm_scale is None:
        sm_scale = d ** -0.5
    torch.cuda.set_device(v.device)
    q8, qs, k8, ks = quantize_qk(q, k)
    o = torch.empty(q.size(), dtype=q.dtype, device=q.device)
    v8, vs = quantize_v(v)
    qattn.qk_int8_sv_f8_accum_f32_fuse_v_scale_attn_inst_buf(q8, k8, v8, o, qs, ks, vs, 0, 0, 2, sm_scale, 0)
    return o
