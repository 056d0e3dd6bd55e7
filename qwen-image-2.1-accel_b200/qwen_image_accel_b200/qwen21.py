"""Qwen-Image 2.1 single-stream block on the sm_100a kernels, with its prefix KV cache.

Mirrors QwenImage21TransformerBlock (WHL:diffusers/models/transformers/
transformer_qwenimage21.py:584-650) in its two modes:

* prefill (`kv_cache_mode="extract"`): the whole joint sequence (text,
  condition images, target image) under the block-causal mask, storing the
  prefix's post-RoPE K/V in a KVLayerCache (:343-353). Prefix tokens take the
  modulation row of t = 0 (the trailing row), target tokens their sample's row
  (_select_modulation_rows, :238-254).
* cached decode (`kv_cache_mode="cached"`): only the target tokens, attending
  to [cached prefix, target] without a mask; this is the reference's fused
  decode block (src/qwen_image_accel/optimizations/fusion.py:38-60 for the
  bf16 profiles, quantized_decode.py:108-137 for the MXFP8 ones): LN x (1+s)
  (MXFP8 straight out of the LN when the projections are MXFP8), Q/K/V
  projections sharing one quantized activation, fused QK-RMSNorm + RoPE +
  prefix pack, Sage attention when the profile has it and nothing is masked,
  gated residual, SwiGLU MLP whose gate/value projections share one
  activation, SwiGLU fused with the MXFP8 quantization of the out projection's
  operand.

Where the reference runs three Q/K/V projections, this runs one over the
stacked [W_q; W_k; W_v] (per-row MXFP8 weight scales, so the codes and every
output are those of the three), normalises and rotates its rows straight into
the joint [prefix, target] K/V buffers behind the copied cache
(qia_qknorm_rope_segment, the same arithmetic as the pack kernel), and in the
MXFP8 profiles takes the attention output as MXFP8 from the attention
epilogue, the gated residuals from the output-projection GEMM epilogues, and
the gate/value projections as one grouped launch -- each byte-identical to
the unfused op sequence it replaces.

As in the reference (quantize_transformer swaps the linears, the MLP forward
is replaced for both modes), the prefill uses the same MXFP8 linears and MLP;
its attention is the reference's per-segment SDPA by default, or, with
`sage_prefill=True`, the tcgen05 Sage kernel with per-query key limits
(qia_sage_attention_prefill).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .kernels.attention import joint_qk_norm_rope
from .kernels.bf16 import swiglu
from .kernels.elementwise import residual
from .kernels.epilogue import layer_norm_scale_quantize, swiglu_quantize
from .kernels.layernorm import layer_norm_scale
from .kernels.mxfp8 import quantize
from .optimizations.mxfp8 import MXFP8Linear, matmul_grouped
from .optimizations.prefill import prefill_attention, segment_prefill_sdpa
from .optimizations.sage_attention import sage_attention, sage_attention_quantized
from .profiles import get_profile


@dataclass(frozen=True)
class Block21Config:
    dim: int = 4096
    heads: int = 32
    head_dim: int = 128
    mlp_ratio: int = 3
    eps: float = 1e-6


def block21_parameter_shapes(cfg: Block21Config) -> dict[str, tuple]:
    """Diffusers state-dict names and shapes of QwenImage21TransformerBlock
    (transformer_qwenimage21.py:584-606; no biases anywhere in 2.1)."""
    d, f, hd = cfg.dim, cfg.dim * cfg.mlp_ratio, cfg.head_dim
    return {
        "attn.to_q.weight": (d, d), "attn.to_k.weight": (d, d), "attn.to_v.weight": (d, d),
        "attn.to_out.0.weight": (d, d), "attn.norm_q.weight": (hd,), "attn.norm_k.weight": (hd,),
        "img_mlp.gate_layer.weight": (f, d), "img_mlp.proj.weight": (f, d), "img_mlp.out.weight": (d, f),
    }


class KVLayerCache:
    """Post-RoPE K and V of the prefix tokens of one block, NHD bf16
    [B, prefix, H, 128] (QwenImage21KVLayerCache, transformer_qwenimage21.py:56-74)."""

    def __init__(self):
        self.k: torch.Tensor | None = None
        self.v: torch.Tensor | None = None

    def store(self, k: torch.Tensor, v: torch.Tensor):
        self.k, self.v = k, v

    def get(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self.k is None:
            raise RuntimeError("KV cache has not been populated yet.")
        return self.k, self.v


class KVCache:
    """One KVLayerCache per block (QwenImage21KVCache, :77-84)."""

    def __init__(self, num_layers: int):
        self.layer_caches = [KVLayerCache() for _ in range(num_layers)]

    def get_layer(self, layer_idx: int) -> KVLayerCache:
        return self.layer_caches[layer_idx]


def modulation_values(modulation: torch.Tensor):
    """The cached decode's per-step vectors from the shared modulation
    [B + 1, 4D] (rows [0, B): the sampled timestep; the trailing row: t = 0,
    which belongs to the cached prefix): (1 + s1, tanh g1, 1 + s2, tanh g2),
    each (B, 1, D) bf16 -- as the reference caches them per modulation tensor
    (fusion.py:45-49)."""
    s1, g1, s2, g2 = modulation[:-1].chunk(4, dim=-1)
    return tuple(t.contiguous() for t in (1 + s1[:, None], g1[:, None].tanh(), 1 + s2[:, None], g2[:, None].tanh()))


class _Norm:
    """The attribute bundle the fused ops read from a norm module (weight, eps,
    normalized_shape, elementwise_affine)."""

    def __init__(self, weight, eps, shape=None):
        self.weight = weight
        self.bias = None
        self.eps = eps
        self.normalized_shape = shape if shape is not None else tuple(weight.shape)
        self.elementwise_affine = False


class Block21:
    """One 2.1 block (params: a name -> tensor mapping or callable with the
    Diffusers names of block21_parameter_shapes).

    Each linear is an MXFP8Linear (tcgen05 block-scaled GEMM) or a bf16
    nn.Linear, chosen per linear: the profile's `quantized` flag sets all of
    them, `quantized=False` keeps a block in bf16 (the profile's skip_blocks),
    and Block21.bind takes whatever modules a caller's model already holds.
    Every fused step is chosen from the types it finds: MXFP8 straight out of
    the LayerNorm when all of its consumers are MXFP8, the attention output as
    MXFP8 into the output projection's gate-residual epilogue when that
    projection is MXFP8, the SwiGLU fused with the quantization of the down
    projection's operand when gate, value and down projections are MXFP8."""

    def __init__(self, params: Callable[[str], torch.Tensor] | dict, cfg: Block21Config = Block21Config(),
                 device="cuda", profile: str = "mxfp8_sage", sage_prefill: bool = False,
                 quantized: bool | None = None):
        prof = get_profile(profile)
        if not prof.fused:
            raise ValueError(f"profile {profile!r} has no fused decode path")
        get = params if callable(params) else params.__getitem__
        mx = prof.quantized if quantized is None else quantized
        dev = torch.device(device)

        def linear(name_or_weight):
            w = get(name_or_weight) if isinstance(name_or_weight, str) else name_or_weight
            w = w.to(dev, torch.bfloat16).contiguous()
            lin = nn.Linear(w.shape[1], w.shape[0], bias=False, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(w)
            return MXFP8Linear(lin) if mx else lin

        self._setup(cfg, prof.sage, sage_prefill,
                    qkv=linear(torch.cat([get(f"attn.to_{n}.weight") for n in "qkv"])),
                    to_out=linear("attn.to_out.0.weight"),
                    mlp=tuple(linear(f"img_mlp.{n}.weight") for n in ("gate_layer", "proj", "out")),
                    norm_q=get("attn.norm_q.weight").to(dev, torch.bfloat16).contiguous(),
                    norm_k=get("attn.norm_k.weight").to(dev, torch.bfloat16).contiguous())

    @classmethod
    def bind(cls, qkv, to_out, mlp, norm_q: torch.Tensor, norm_k: torch.Tensor, cfg: Block21Config, sage: bool,
             sage_prefill: bool = False) -> "Block21":
        """A Block21 over modules a caller already holds, sharing their
        weights: qkv is one linear over the stacked [W_q; W_k; W_v] rows or a
        (to_q, to_k, to_v) tuple; to_out, mlp = (gate_layer, proj, out) are
        nn.Linear (bf16, no bias) or MXFP8Linear modules."""
        self = cls.__new__(cls)
        self._setup(cfg, sage, sage_prefill, qkv=qkv, to_out=to_out, mlp=tuple(mlp), norm_q=norm_q, norm_k=norm_k)
        return self

    def _setup(self, cfg, sage, sage_prefill, qkv, to_out, mlp, norm_q, norm_k):
        self.cfg = cfg
        self.sage, self.sage_prefill = sage, sage_prefill
        self.qkv, self.to_out = qkv, to_out
        self.gate_layer, self.proj, self.out = mlp
        self.norm_q = _Norm(norm_q, cfg.eps)
        self.norm_k = _Norm(norm_k, cfg.eps)
        self.norm = _Norm(None, cfg.eps, (cfg.dim,))          # img_norm1 / img_norm2: no affine
        parts = qkv if isinstance(qkv, tuple) else (qkv,)
        self.qkv_mx = all(isinstance(p, MXFP8Linear) for p in parts)
        self.out_mx = isinstance(to_out, MXFP8Linear)
        self.gv_mx = isinstance(self.gate_layer, MXFP8Linear) and isinstance(self.proj, MXFP8Linear)
        self.down_mx = isinstance(self.out, MXFP8Linear)

    @property
    def quantized(self) -> bool:
        """Every linear of the block is MXFP8."""
        return self.qkv_mx and self.out_mx and self.gv_mx and self.down_mx

    # ------------------------------------------------------------------ helpers
    def _normalized(self, h, scale, mx: bool):
        """LN(h) x scale, as MXFP8 straight out of the LN when its consumers
        are MXFP8 linears (mx), else bf16."""
        if not mx:
            return layer_norm_scale(h, scale, self.norm)
        x = layer_norm_scale_quantize(h, scale, self.norm)
        if x is None:
            raise NotImplementedError(f"LN + MXFP8: unsupported input {tuple(h.shape)}")
        return x

    @staticmethod
    def _apply(lin, x):
        """One linear on x: an MXFP8 activation (Quantized) or a bf16 tensor."""
        if isinstance(lin, MXFP8Linear):
            if isinstance(x, torch.Tensor):
                x = quantize(x.reshape(-1, x.shape[-1]).contiguous())
            return lin.matmul(x)
        return F.linear(x, lin.weight)

    def _qkv_into(self, x, b, s, freqs, oq, ok, ov, offset):
        """q|k|v projection of the LN output x (bf16 tensor, or MXFP8 Quantized
        when the projections are MXFP8) for s tokens per sample, RMS-normalised
        and rotated into rows [offset, offset + s) of the joint NHD buffers."""
        if isinstance(self.qkv, tuple):
            qkv = torch.cat([self._apply(p, x).view(b, s, -1) for p in self.qkv], dim=-1)
        else:
            qkv = self._apply(self.qkv, x).view(b, s, -1)
        joint_qk_norm_rope(qkv, self.norm_q.weight, self.norm_k.weight, torch.view_as_real(freqs).contiguous(),
                           oq, ok, ov, offset, eps=self.cfg.eps)

    def _joint(self, b, total, device):
        shape = (b, total, self.cfg.heads, self.cfg.head_dim)
        return tuple(torch.empty(shape, device=device, dtype=torch.bfloat16) for _ in range(3))

    def _out_proj(self, attn):
        return self._apply(self.to_out, attn.flatten(2, 3).contiguous()).view(*attn.shape[:2], -1)

    def _swiglu_act(self, x):
        """MXFP8 SwiGLU activation of the MLP (gate, value and down projections
        MXFP8): the gate and value projections of one shared activation in one
        grouped launch, then SwiGLU + quantization in one pass. (The
        single-GEMM form with the SwiGLU in the epilogue,
        MXFP8Linear.matmul_swiglu_quantize, gives the same bytes but measured
        slower here: its per-element IEEE divide and exp hold the accumulator
        hand-off of the GEMM.)"""
        a = x if not isinstance(x, torch.Tensor) else quantize(x.reshape(-1, x.shape[-1]).contiguous())
        gate, value = matmul_grouped([(self.gate_layer, a), (self.proj, a)])
        return swiglu_quantize(gate, value)

    def _gate_value(self, x):
        if self.gv_mx:
            a = x if not isinstance(x, torch.Tensor) else quantize(x.reshape(-1, x.shape[-1]).contiguous())
            return matmul_grouped([(self.gate_layer, a), (self.proj, a)])
        return self._apply(self.gate_layer, x), self._apply(self.proj, x)

    def _mlp(self, x, lead):
        """SwiGLU MLP; x is the LN output (bf16, or its MXFP8 quantization when
        the gate and value projections are MXFP8)."""
        if self.gv_mx and self.down_mx:
            return self.out.matmul(self._swiglu_act(x)).view(*lead, -1)
        gate, value = self._gate_value(x)
        return self._apply(self.out, swiglu(gate.contiguous(), value.contiguous())).view(*lead, -1)

    def _rows(self, name, x, vectors, prefix_len, other=None):
        """LN x (1+s) (name "ln") or the gated residual (name "res") with the
        prefix rows of every sample using vector row B (t = 0) and the target
        rows vector row b: one launch per row range, into one output."""
        b, s, d = x.shape
        out = torch.empty_like(x)
        xf, of = x.view(-1, d), out.view(-1, d)
        yf = other.view(-1, d) if other is not None else None
        st = _lib.stream(x.device)
        for bi in range(b):
            for r0, r1, vec in ((0, prefix_len, b), (prefix_len, s, bi)):
                n = r1 - r0
                if n <= 0:
                    continue
                lo = bi * s + r0
                v = vectors[vec:vec + 1]
                if name == "ln":
                    _lib.call("qia_ln_mod", _lib.ptr(xf[lo:lo + n]), _lib.ptr(v), None, _lib.ptr(of[lo:lo + n]), n, d,
                              n, float(self.cfg.eps), st)
                else:
                    _lib.call("qia_gated_residual", _lib.ptr(xf[lo:lo + n]), _lib.ptr(yf[lo:lo + n]), _lib.ptr(v),
                              _lib.ptr(of[lo:lo + n]), n, d, n, st)
        return out

    # ------------------------------------------------------------------ modes
    def forward_cached(self, h: torch.Tensor, values, freqs: torch.Tensor, layer_cache: KVLayerCache,
                       key_valid: torch.Tensor | None = None) -> torch.Tensor:
        """Cached decode of the target tokens h [B, St, D]; values =
        modulation_values(modulation); freqs complex64 [St, 64] (the target's
        rows of the RoPE table); key_valid bool [B, prefix + St] or None."""
        s1, g1, s2, g2 = values
        b, st, _ = h.shape
        h = h.contiguous()
        cached_k, cached_v = layer_cache.get()
        p = cached_k.shape[1]
        if cached_k.shape[0] != b or cached_v.shape != cached_k.shape:
            raise ValueError("cached decode: the cache does not match the batch")
        oq, ok, ov = self._joint(b, p + st, h.device)
        ok[:, :p].copy_(cached_k)
        ov[:, :p].copy_(cached_v)
        self._qkv_into(self._normalized(h, s1, self.qkv_mx), b, st, freqs, oq, ok, ov, p)
        q = oq[:, p:]
        if self.sage and key_valid is None and self.out_mx:
            h = self.to_out.matmul_gate_residual(sage_attention_quantized(q, ok, ov), g1, h)
        else:
            if self.sage and key_valid is None:
                attn = sage_attention(q, ok, ov)
            else:
                mask = None if key_valid is None else key_valid[:, None, None, :]
                attn = F.scaled_dot_product_attention(q.transpose(1, 2), ok.transpose(1, 2), ov.transpose(1, 2),
                                                      attn_mask=mask).transpose(1, 2)
            h = residual(h, self._out_proj(attn).contiguous(), g1)
        x = self._normalized(h, s2, self.gv_mx)
        if self.gv_mx and self.down_mx:
            return self.out.matmul_gate_residual(self._swiglu_act(x), g2, h)
        return residual(h, self._mlp(x, (b, st)).contiguous(), g2)

    def attention_cached(self, x, freqs: torch.Tensor, layer_cache: KVLayerCache,
                         key_valid: torch.Tensor | None = None) -> torch.Tensor:
        """The attention half of the cached decode on an already modulated
        input x [B, St, D] bf16: Q/K/V projections, QK-RMSNorm + RoPE behind the
        cached prefix K/V, attention over [prefix, target] (Sage when the block
        has it and nothing is masked, else SDPA), output projection -> bf16
        [B, St, D]."""
        b, st, _ = x.shape
        cached_k, cached_v = layer_cache.get()
        p = cached_k.shape[1]
        oq, ok, ov = self._joint(b, p + st, x.device)
        ok[:, :p].copy_(cached_k)
        ov[:, :p].copy_(cached_v)
        self._qkv_into(x.contiguous(), b, st, freqs, oq, ok, ov, p)
        q = oq[:, p:]
        if self.sage and key_valid is None:
            attn = sage_attention(q, ok, ov)
        else:
            mask = None if key_valid is None else key_valid[:, None, None, :]
            attn = F.scaled_dot_product_attention(q.transpose(1, 2), ok.transpose(1, 2), ov.transpose(1, 2),
                                                  attn_mask=mask).transpose(1, 2)
        return self._out_proj(attn)

    def forward_prefill(self, h: torch.Tensor, modulation: torch.Tensor, freqs: torch.Tensor,
                        image_ids: torch.Tensor, prefix_len: int, layer_cache: KVLayerCache | None = None,
                        key_valid: torch.Tensor | None = None) -> torch.Tensor:
        """Prefill of the joint sequence h [B, S, D] (target image = the last
        S - prefix_len tokens); modulation [B + 1, 4D]; freqs complex64
        [S, 64]; image_ids int [S] (-1 at text tokens). Stores the prefix's
        post-RoPE K/V in layer_cache when given (kv_cache_mode="extract")."""
        b, s, _ = h.shape
        h = h.contiguous()
        s1, g1, s2, g2 = modulation.chunk(4, dim=-1)
        one_s1, tanh_g1, one_s2, tanh_g2 = ((1 + s1).contiguous(), g1.tanh().contiguous(),
                                            (1 + s2).contiguous(), g2.tanh().contiguous())
        x = self._rows("ln", h, one_s1, prefix_len)
        q, k, v = self._joint(b, s, h.device)
        self._qkv_into(x, b, s, freqs, q, k, v, 0)
        if layer_cache is not None:
            layer_cache.store(k[:, :prefix_len].clone(), v[:, :prefix_len].clone())
        if self.sage_prefill:
            attn = prefill_attention(q, k, v, image_ids, key_valid=key_valid)
        else:
            attn = segment_prefill_sdpa(q, k, v, image_ids, prefix_len, key_valid=key_valid)
        h = self._rows("res", h, tanh_g1, prefix_len, other=self._out_proj(attn).contiguous())
        x = self._rows("ln", h, one_s2, prefix_len)
        return self._rows("res", h, tanh_g2, prefix_len, other=self._mlp(x, (b, s)).contiguous())
