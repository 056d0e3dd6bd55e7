"""Sage-style INT8/FP8 joint attention on tcgen05 (decode path of the sage profiles).

Mirrors src/qwen_image_accel/optimizations/sage_attention.py: the
`qw21::sage_decode(q, k, v)` custom op (NHD bf16 in, NHD bf16 out) and the
QW21_SAGE_ACCUM / QW21_SAGE_QK_GRAN settings, now served by the sm_100a
kernels in libqia_b200.so instead of the SageAttention2 extension. The only
accumulation implemented is the reference default "fp32+fp32" and the only
granularity "per_warp"; other values raise.
"""
from __future__ import annotations

import ctypes
import os

import torch

from .. import _lib

ACCUM = os.environ.get("QW21_SAGE_ACCUM", "fp32+fp32").strip()
QK_GRAN = os.environ.get("QW21_SAGE_QK_GRAN", "per_warp").strip()


def _check_settings():
    if ACCUM != "fp32+fp32" or QK_GRAN != "per_warp":
        raise NotImplementedError("only QW21_SAGE_ACCUM=fp32+fp32 and QW21_SAGE_QK_GRAN=per_warp are implemented")


def workspace_bytes(batch: int, heads: int, seq_q: int, seq_kv: int) -> int:
    n = _lib.load().qia_sage_workspace_bytes(batch, heads, seq_q, seq_kv)
    if n < 0:
        raise ValueError("bad attention sizes")
    return int(n)


def _pad128(s):
    return (s + 127) // 128 * 128


def workspace_views(ws: torch.Tensor, batch: int, heads: int, seq_q: int, seq_kv: int) -> dict:
    """Typed views of the workspace regions (same layout as the C side)."""
    bh, sqp, skp = batch * heads, _pad128(seq_q), _pad128(seq_kv)
    regions = [("q8", bh * sqp * 128, torch.int8, (bh, sqp, 128)),
               ("k8", bh * skp * 128, torch.int8, (bh, skp, 128)),
               ("v8", bh * skp * 128, torch.float8_e4m3fn, (bh, skp, 128)),
               ("q_scale", bh * (sqp // 32) * 4, torch.float32, (bh, sqp // 32)),
               ("k_scale", bh * (skp // 64) * 4, torch.float32, (bh, skp // 64)),
               ("v_scale", bh * 128 * 4, torch.float32, (bh, 128)),
               ("k_mean", bh * 128 * 2, torch.bfloat16, (bh, 128)),
               ("v_recp", bh * 128 * 4, torch.float32, (bh, 128)),
               ("k_part", bh * (skp // 32) * 128 * 4, torch.float32, (bh, skp // 32, 128)),
               ("v_part", bh * (skp // 32) * 128 * 4, torch.float32, (bh, skp // 32, 128)),
               ("kn", bh * skp * 128 * 2, torch.bfloat16, (bh, skp, 128))]
    out, off = {}, 0
    for name, nbytes, dtype, shape in regions:
        out[name] = ws[off:off + nbytes].view(dtype).view(shape)
        off += (nbytes + 255) // 256 * 256
    return out


def _strides(*ts):
    vals = []
    for t in ts:
        if t.stride(-1) != 1:
            raise NotImplementedError("head_dim must be contiguous")
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * len(vals))(*vals)


def _validate(q, k, v):
    _lib.require_cuda(q, k, v)
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
        raise NotImplementedError("expects NHD q (B, Sq, H, 128) and k/v (B, Skv, H, 128)")
    if q.shape[-1] != 128 or any(t.dtype != torch.bfloat16 for t in (q, k, v)):
        raise NotImplementedError("expects bf16 tensors with head_dim 128")


def sage_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float | None = None,
                   out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Sage-style attention: INT8 Q.K^T (K smoothed), FP8 P.V, NHD bf16 in and out."""
    _check_settings()
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    if out is None:
        out = torch.empty_like(q)
    need = workspace_bytes(b, h, sq, skv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    _lib.call("qia_sage_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), b, sq, skv, h, d,
              _strides(q, k, v, out), float(sm_scale or 0.0), _lib.ptr(workspace), workspace.numel(),
              _lib.stream(q.device))
    return out


def sage_attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_limit: torch.Tensor,
                           sm_scale: float | None = None, out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """sage_attention where query token t sees keys [0, kv_limit[t]) only
    (kv_limit int32 [Sq], shared by the batch, or [B, Sq]); the block-causal
    prefill of the 2.1 prefix-KV path (see prefill.prefill_attention)."""
    _check_settings()
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    _lib.require_cuda(kv_limit)
    if kv_limit.dtype != torch.int32 or kv_limit.shape[-1] != sq or kv_limit.ndim not in (1, 2) \
            or kv_limit.stride(-1) != 1 or (kv_limit.ndim == 2 and kv_limit.shape[0] != b):
        raise NotImplementedError("kv_limit must be int32 [Sq] or [B, Sq] with a contiguous last dim")
    stride_b = 0 if kv_limit.ndim == 1 or b == 1 else kv_limit.stride(0)
    if out is None:
        out = torch.empty_like(q)
    need = workspace_bytes(b, h, sq, skv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    _lib.call("qia_sage_attention_prefill", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out), _lib.ptr(kv_limit),
              stride_b, b, sq, skv, h, d, _strides(q, k, v, out), float(sm_scale or 0.0), _lib.ptr(workspace),
              workspace.numel(), _lib.stream(q.device))
    return out


def sage_attention_split(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, split: int, out_a: torch.Tensor,
                         out_b: torch.Tensor, sm_scale: float | None = None,
                         workspace: torch.Tensor | None = None) -> None:
    """Joint attention whose query tokens [0, split) land in out_a and
    [split, Sq) in out_b (both NHD bf16), e.g. the text and image streams."""
    _check_settings()
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    need = workspace_bytes(b, h, sq, skv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    _lib.call("qia_sage_attention_split", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out_a), _lib.ptr(out_b),
              split, b, sq, skv, h, d, _strides(q, k, v, out_a, out_b), float(sm_scale or 0.0), _lib.ptr(workspace),
              workspace.numel(), _lib.stream(q.device))


def sage_attention_split_quantized(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, split: int,
                                   sm_scale: float | None = None, workspace: torch.Tensor | None = None):
    """sage_attention_split whose two outputs come back as MXFP8 activations
    (Quantized, rows = batch * stream tokens, K = heads * 128) ready for the
    output projections: byte-identical to quantize() of the bf16 outputs."""
    from ..kernels.mxfp8 import empty_quantized
    _check_settings()
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    need = workspace_bytes(b, h, sq, skv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    qa = empty_quantized(b * split, h * d, q.device)
    qb = empty_quantized(b * (sq - split), h * d, q.device)
    for t in (qa, qb):             # rows past the live ones (padding to 128) stay zero
        if t.values.shape[0] > t.rows:
            t.values[t.rows:].view(torch.uint8).zero_()
            t.scales.view(torch.uint8).zero_()
    _lib.call("qia_sage_attention_split_mx", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(qa.values),
              _lib.ptr(qa.scales), _lib.ptr(qb.values), _lib.ptr(qb.scales), split, b, sq, skv, h, d,
              _strides(q, k, v), float(sm_scale or 0.0), _lib.ptr(workspace), workspace.numel(),
              _lib.stream(q.device))
    return qa, qb


def sage_attention_quantized(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float | None = None,
                             workspace: torch.Tensor | None = None):
    """sage_attention whose output comes back as one MXFP8 activation
    (Quantized, rows = batch * Sq, K = heads * 128) for the output projection:
    byte-identical to quantize() of the bf16 output (qia_sage_attention_split_mx
    with split = Sq). q may be a strided view (e.g. the target rows of a joint
    [prefix, target] buffer)."""
    from ..kernels.mxfp8 import empty_quantized
    _check_settings()
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    need = workspace_bytes(b, h, sq, skv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    qa = empty_quantized(b * sq, h * d, q.device)
    if qa.values.shape[0] > qa.rows:      # rows past the live ones (padding to 128) stay zero
        qa.values[qa.rows:].view(torch.uint8).zero_()
        qa.scales.view(torch.uint8).zero_()
    _lib.call("qia_sage_attention_split_mx", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(qa.values),
              _lib.ptr(qa.scales), None, None, sq, b, sq, skv, h, d, _strides(q, k, v), float(sm_scale or 0.0),
              _lib.ptr(workspace), workspace.numel(), _lib.stream(q.device))
    return qa


def _joint_args(qkv0, qkv1, weights0, weights1, freqs0, freqs1, heads):
    """Pointer/size arguments of the joint entries (see sage_quantize_joint)."""
    _lib.require_cuda(qkv0, qkv1, *weights0, *weights1, freqs0, freqs1)
    for t in (qkv0, qkv1):
        if t.ndim != 3 or t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.stride(0) != t.shape[1] * t.stride(1):
            raise NotImplementedError("qkv projections must be (B, L, >= 3*H*128) bf16 with evenly strided rows")
        if t.shape[2] < 3 * heads * 128:
            raise ValueError("qkv projection narrower than 3*heads*128")
    if qkv0.shape[0] != qkv1.shape[0]:
        raise ValueError("the two streams' batch sizes differ")
    for f, t in ((freqs0, qkv0), (freqs1, qkv1)):
        if f.dtype != torch.float32 or not f.is_contiguous() or f.numel() < t.shape[1] * 128:
            raise NotImplementedError("freqs must be contiguous float32 (L, 64, 2)")
    for w in (*weights0, *weights1):
        if w.dtype != torch.bfloat16 or w.numel() != 128 or not w.is_contiguous():
            raise NotImplementedError("norm weights must be contiguous bf16 [128]")
    return [_lib.ptr(qkv0), qkv0.stride(1), _lib.ptr(qkv1), qkv1.stride(1), _lib.ptr(weights0[0]),
            _lib.ptr(weights0[1]), _lib.ptr(weights1[0]), _lib.ptr(weights1[1]), _lib.ptr(freqs0), _lib.ptr(freqs1)]


def sage_quantize_joint(qkv0: torch.Tensor, qkv1: torch.Tensor, weights0, weights1, freqs0: torch.Tensor,
                        freqs1: torch.Tensor, heads: int, eps: float = 1e-6) -> dict:
    """The quantization half for the joint [stream 0, stream 1] sequence, read
    straight from the streams' fused q|k|v projections (B, L_i, 3*H*128) with
    each stream's QK-RMSNorm (weights_i = (norm_q, norm_k)) and RoPE (freqs_i
    float32 (L_i, 64, 2)) applied on load. The workspace equals
    joint_qk_norm_rope on both streams followed by sage_quantize."""
    b, l0, l1 = qkv0.shape[0], qkv0.shape[1], qkv1.shape[1]
    args = _joint_args(qkv0, qkv1, weights0, weights1, freqs0, freqs1, heads)
    s = l0 + l1
    need = workspace_bytes(b, heads, s, s)
    ws = torch.empty(need, device=qkv0.device, dtype=torch.uint8)
    _lib.call("qia_sage_quantize_joint", *args, b, l0, l1, heads, 128, float(eps), _lib.ptr(ws), need,
              _lib.stream(qkv0.device))
    views = workspace_views(ws, b, heads, s, s)
    views["_workspace"] = ws
    return views


def sage_attention_joint_quantized(qkv0: torch.Tensor, qkv1: torch.Tensor, weights0, weights1,
                                   freqs0: torch.Tensor, freqs1: torch.Tensor, heads: int, eps: float = 1e-6,
                                   sm_scale: float | None = None, workspace: torch.Tensor | None = None):
    """Joint attention of the dual-stream block from the two streams' fused
    q|k|v projections (QK-RMSNorm + RoPE + Sage quantization fused), with the
    per-stream outputs as MXFP8 activations (Quantized, rows = batch * L_i,
    K = heads * 128): equal to joint_qk_norm_rope on both streams followed by
    sage_attention_split_quantized(q, k, v, L_0)."""
    from ..kernels.mxfp8 import empty_quantized
    _check_settings()
    b, l0, l1 = qkv0.shape[0], qkv0.shape[1], qkv1.shape[1]
    args = _joint_args(qkv0, qkv1, weights0, weights1, freqs0, freqs1, heads)
    s = l0 + l1
    need = workspace_bytes(b, heads, s, s)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=qkv0.device, dtype=torch.uint8)
    qa = empty_quantized(b * l0, heads * 128, qkv0.device)
    qb = empty_quantized(b * l1, heads * 128, qkv0.device)
    for t in (qa, qb):             # rows past the live ones (padding to 128) stay zero
        if t.values.shape[0] > t.rows:
            t.values[t.rows:].view(torch.uint8).zero_()
            t.scales.view(torch.uint8).zero_()
    _lib.call("qia_sage_attention_joint_mx", *args, _lib.ptr(qa.values), _lib.ptr(qa.scales), _lib.ptr(qb.values),
              _lib.ptr(qb.scales), b, l0, l1, heads, 128, float(eps), float(sm_scale or 0.0), _lib.ptr(workspace),
              workspace.numel(), _lib.stream(qkv0.device))
    return qa, qb


def sage_attention_from_workspace(workspace: torch.Tensor, out: torch.Tensor,
                                  sm_scale: float | None = None) -> torch.Tensor:
    """The attention half alone (qia_sage_attn_quantized) on a workspace that
    sage_quantize or sage_quantize_joint filled for out's (B, S, H) with
    S = Sq = Skv: out (B, S, H, 128) bf16, any strides with a contiguous
    head_dim; returns out."""
    _check_settings()
    _lib.require_cuda(workspace, out)
    if out.ndim != 4 or out.shape[-1] != 128 or out.dtype != torch.bfloat16:
        raise NotImplementedError("out must be (B, S, H, 128) bf16")
    b, s, h, d = out.shape
    need = workspace_bytes(b, h, s, s)
    if workspace.dtype != torch.uint8 or workspace.numel() < need:
        raise ValueError(f"workspace holds {workspace.numel()} bytes, the attention needs {need}")
    _lib.call("qia_sage_attn_quantized", _lib.ptr(workspace), _lib.ptr(out), b, s, s, h, d, _strides(out),
              float(sm_scale or 0.0), _lib.stream(out.device))
    return out


def sage_quantize(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> dict:
    """Run only the quantization half; returns the workspace views."""
    _validate(q, k, v)
    b, sq, h, d = q.shape
    skv = k.shape[1]
    need = workspace_bytes(b, h, sq, skv)
    ws = torch.empty(need, device=q.device, dtype=torch.uint8)
    _lib.call("qia_sage_quantize", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), b, sq, skv, h, d, _strides(q, k, v),
              _lib.ptr(ws), need, _lib.stream(q.device))
    views = workspace_views(ws, b, h, sq, skv)
    views["_workspace"] = ws
    return views


@torch.library.custom_op("qw21::sage_decode", mutates_args=())
def sage_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return sage_attention(q, k, v)


@sage_decode.register_fake
def _(q, k, v):
    return torch.empty_like(q)
