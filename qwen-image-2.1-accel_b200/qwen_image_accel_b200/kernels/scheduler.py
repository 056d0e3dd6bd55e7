"""True-CFG combine + flow-match Euler update (qia_cfg_euler, qia_cfg_euler_sched),
and the same fused behind the proj_out GEMM (qia_proj_out_cfg_euler).

Eager form (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
schedulers/scheduling_flow_match_euler_discrete.py:483-517):
    comb = neg + s * (cond - neg)
    v = comb * (||cond|| / ||comb||)          (norms over the last dim)
    out = (latents.float() + (sigma_next - sigma) * v).to(latents.dtype)
"""
from __future__ import annotations

import torch

from .. import _lib


def _check_sigmas(sigmas: torch.Tensor):
    if sigmas.dtype != torch.float32 or sigmas.numel() < 2 or not sigmas.is_contiguous():
        raise ValueError("sigmas: a contiguous float32 device tensor holding (sigma, sigma_next)")


def cfg_euler(cond: torch.Tensor, neg: torch.Tensor, latents: torch.Tensor, cfg_scale: float,
              dt: float | None = None, out: torch.Tensor | None = None,
              sigmas: torch.Tensor | None = None) -> torch.Tensor:
    """cond, neg, latents: bf16 of one shape (rows x dim in the last axis);
    returns the updated latents (bf16). The step is `dt` (a host float) or,
    given `sigmas` (device float32 (sigma, sigma_next)), sigma_next - sigma
    taken on the device."""
    _lib.require_cuda(cond, neg, latents, sigmas)
    if not (cond.shape == neg.shape == latents.shape) or any(
            t.dtype != torch.bfloat16 or not t.is_contiguous() for t in (cond, neg, latents)):
        raise NotImplementedError("cfg_euler: contiguous bf16 cond/neg/latents of one shape")
    if (dt is None) == (sigmas is None):
        raise ValueError("cfg_euler: give exactly one of dt and sigmas")
    if out is None:
        out = torch.empty_like(latents)
    dim = latents.shape[-1]
    if sigmas is None:
        _lib.call("qia_cfg_euler", _lib.ptr(cond), _lib.ptr(neg), _lib.ptr(latents), _lib.ptr(out),
                  latents.numel() // dim, dim, float(cfg_scale), float(dt), _lib.stream(latents.device))
    else:
        _check_sigmas(sigmas)
        _lib.call("qia_cfg_euler_sched", _lib.ptr(cond), _lib.ptr(neg), _lib.ptr(latents), _lib.ptr(out),
                  latents.numel() // dim, dim, float(cfg_scale), _lib.ptr(sigmas), _lib.stream(latents.device))
    return out


def proj_out_cfg_euler(y: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, latents: torch.Tensor,
                       cfg_scale: float, sigmas: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The step's tail in one launch: y [2 * B, S, K] bf16 (the CFG batch's
    norm_out output: B conditional rows, then B unconditional), proj_out
    weight [64, K] / bias [64]; latents [B, S, 64]; sigmas device float32
    (sigma, sigma_next). Returns the updated latents (out may be latents)."""
    _lib.require_cuda(y, weight, bias, latents, sigmas)
    _check_sigmas(sigmas)
    n, k = weight.shape
    rows = latents.numel() // n
    if (y.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or latents.dtype != torch.bfloat16
            or not y.is_contiguous() or not weight.is_contiguous() or not latents.is_contiguous()
            or y.numel() != 2 * rows * k or latents.shape[-1] != n or (bias is not None and bias.numel() != n)):
        raise NotImplementedError("proj_out_cfg_euler: contiguous bf16 y [2B, S, K], weight [64, K], "
                                  "latents [B, S, 64]")
    if out is None:
        out = torch.empty_like(latents)
    _lib.call("qia_proj_out_cfg_euler", _lib.ptr(y), _lib.ptr(weight), _lib.ptr(bias), _lib.ptr(latents),
              _lib.ptr(out), rows, k, n, float(cfg_scale), _lib.ptr(sigmas), _lib.stream(latents.device))
    return out
