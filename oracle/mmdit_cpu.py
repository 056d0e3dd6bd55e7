"""Eager CPU restatement of the dual-stream (v1) MMDiT block -- TEST/BASELINE ONLY.

The reference runs this model as eager BF16 PyTorch (the Diffusers module,
WHL:diffusers/models/transformers/transformer_qwenimage.py:633-790 for the
block, :479-601 for the joint attention processor). This file restates that
forward pass in plain torch ops on the host CPU. It is used by bench.py's
cpu_baseline leg and `--impl reference` arm (the reference's CPU path timed
on the box's host cores) and by tests as a checker; the product never calls
it.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _rms(x, w, eps):
    var = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    return (x * torch.rsqrt(var + eps)).to(w.dtype) * w


def _rope(x, freqs_c):
    xr = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xr * freqs_c.unsqueeze(1)).flatten(3).type_as(x)


def block_forward(p: dict, prefix: str, x: torch.Tensor, c: torch.Tensor, temb: torch.Tensor,
                  img_freqs: torch.Tensor, txt_freqs: torch.Tensor, heads: int, eps: float = 1e-6):
    """One QwenImageTransformerBlock forward (no masks), eager bf16.

    p: state-dict tensors keyed by Diffusers names; img/txt freqs complex64."""
    W = lambda n: p[prefix + n]  # noqa: E731
    D = x.shape[-1]
    img_mod = F.linear(F.silu(temb), W("img_mod.1.weight"), W("img_mod.1.bias"))
    txt_mod = F.linear(F.silu(temb), W("txt_mod.1.weight"), W("txt_mod.1.bias"))
    im1, im2 = img_mod.chunk(2, dim=-1)
    tm1, tm2 = txt_mod.chunk(2, dim=-1)

    def modulate(h, m):
        shift, scale, gate = m.chunk(3, dim=-1)
        return h * (1 + scale.unsqueeze(1)) + shift.unsqueeze(1), gate.unsqueeze(1)

    xm, g1 = modulate(F.layer_norm(x, (D,), eps=eps), im1)
    cm, tg1 = modulate(F.layer_norm(c, (D,), eps=eps), tm1)
    lin = lambda h, n: F.linear(h, W(n + ".weight"), W(n + ".bias"))  # noqa: E731
    hd = D // heads
    iq, ik, iv = (lin(xm, "attn." + n).unflatten(-1, (-1, hd)) for n in ("to_q", "to_k", "to_v"))
    tq, tk, tv = (lin(cm, "attn." + n).unflatten(-1, (-1, hd)) for n in ("add_q_proj", "add_k_proj", "add_v_proj"))
    iq, ik = _rms(iq, W("attn.norm_q.weight"), eps), _rms(ik, W("attn.norm_k.weight"), eps)
    tq, tk = _rms(tq, W("attn.norm_added_q.weight"), eps), _rms(tk, W("attn.norm_added_k.weight"), eps)
    iq, ik = _rope(iq, img_freqs), _rope(ik, img_freqs)
    tq, tk = _rope(tq, txt_freqs), _rope(tk, txt_freqs)
    q, k, v = torch.cat([tq, iq], 1), torch.cat([tk, ik], 1), torch.cat([tv, iv], 1)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    o = o.flatten(2, 3).to(q.dtype)
    lt = c.shape[1]
    x = x + g1 * lin(o[:, lt:].contiguous(), "attn.to_out.0")
    c = c + tg1 * lin(o[:, :lt].contiguous(), "attn.to_add_out")
    xm2, g2 = modulate(F.layer_norm(x, (D,), eps=eps), im2)
    x = x + g2 * lin(F.gelu(lin(xm2, "img_mlp.net.0.proj"), approximate="tanh"), "img_mlp.net.2")
    cm2, tg2 = modulate(F.layer_norm(c, (D,), eps=eps), tm2)
    c = c + tg2 * lin(F.gelu(lin(cm2, "txt_mlp.net.0.proj"), approximate="tanh"), "txt_mlp.net.2")
    return x, c


def model_forward(p: dict, cfg, x: torch.Tensor, enc: torch.Tensor, timestep: torch.Tensor, img_freqs, txt_freqs):
    """Whole QwenImageTransformer2DModel forward (eager), using block_forward.
    img/txt freqs complex64; cfg: an MMDiTConfig-like object."""
    from math import log

    L = lambda n, h: F.linear(h, p[n + ".weight"], p[n + ".bias"])  # noqa: E731
    h = L("img_in", x)
    t = timestep.to(torch.bfloat16)
    c = L("txt_in", _rms(enc, p["txt_norm.weight"], cfg.eps))
    half = 128
    exponent = -log(10000) * torch.arange(0, half, dtype=torch.float32) / half
    emb = 1000 * (t[:, None].float() * torch.exp(exponent)[None, :])
    emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
    emb = torch.cat([emb[:, half:], emb[:, :half]], dim=-1).to(torch.bfloat16)
    te = "time_text_embed.timestep_embedder."
    temb = L(te + "linear_2", F.silu(L(te + "linear_1", emb)))
    for i in range(cfg.num_layers):
        c, h = block_forward(p, f"transformer_blocks.{i}.", h, c, temb, img_freqs, txt_freqs,
                             cfg.num_attention_heads, cfg.eps)[::-1]
    e = L("norm_out.linear", F.silu(temb))
    scale, shift = e.chunk(2, dim=1)
    h = F.layer_norm(h, (h.shape[-1],), eps=cfg.eps) * (1 + scale)[:, None, :] + shift[:, None, :]
    return L("proj_out", h)
