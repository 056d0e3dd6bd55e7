"""True-CFG combine + flow-match Euler update in one launch (qia_cfg_euler).

Eager form (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
schedulers/scheduling_flow_match_euler_discrete.py:483-517):
    comb = neg + s * (cond - neg)
    v = comb * (||cond|| / ||comb||)          (norms over the last dim)
    out = (latents.float() + (sigma_next - sigma) * v).to(latents.dtype)
"""
from __future__ import annotations

import torch

from .. import _lib


def cfg_euler(cond: torch.Tensor, neg: torch.Tensor, latents: torch.Tensor, cfg_scale: float, dt: float,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """cond, neg, latents: bf16 of one shape (rows x dim in the last axis);
    returns the updated latents (bf16)."""
    _lib.require_cuda(cond, neg, latents)
    if not (cond.shape == neg.shape == latents.shape) or any(
            t.dtype != torch.bfloat16 or not t.is_contiguous() for t in (cond, neg, latents)):
        raise NotImplementedError("cfg_euler: contiguous bf16 cond/neg/latents of one shape")
    if out is None:
        out = torch.empty_like(latents)
    dim = latents.shape[-1]
    _lib.call("qia_cfg_euler", _lib.ptr(cond), _lib.ptr(neg), _lib.ptr(latents), _lib.ptr(out),
              latents.numel() // dim, dim, float(cfg_scale), float(dt), _lib.stream(latents.device))
    return out
