"""Dual-stream MMDiT denoise step (the Qwen-Image v1 layout) on the sm_100a kernels.

The model is the one BASELINE configs 4-5 describe and the pinned Diffusers
wheel defines (WHL:diffusers/models/transformers/transformer_qwenimage.py:
QwenImageTransformer2DModel / QwenImageTransformerBlock, :633-790, :859-1031):
60 dual-stream blocks, hidden 3072, 24x128 heads, FFN 12288 GELU-tanh with
biases, AdaLN shift/scale/gate, text 3584 -> 3072. Weights use the Diffusers
state-dict names, so a checkpoint of that model loads as is.

Per block the hot path is (the image and text streams' LayerNorms and the
GEMMs of each projection share their shapes' inner dimensions and run as one
grouped launch each, text rows/tiles last):
  LN + (1+scale), +shift -> MXFP8         qia_ln_mod_quant_grouped
  fused Q|K|V GEMM (+bias)                 qia_mxfp8_gemm_grouped (bf16)
  QK-RMSNorm + RoPE + Sage quantization    qia_sage_attention_joint_mx (both
    + joint [txt, img] INT8/FP8 attention    streams' projections in, per-stream
    -> MXFP8                                 MXFP8 attention outputs back)
  out-proj GEMM + gate + residual          qia_mxfp8_gemm_grouped (gate-residual)
  LN + (1+scale), +shift -> MXFP8          qia_ln_mod_quant_grouped
  FFN up GEMM + bias + GELU -> MXFP8       qia_mxfp8_gemm_grouped (GELU-quant)
  FFN down GEMM + gate + residual          qia_mxfp8_gemm_grouped (gate-residual)
The prologue/epilogue layers outside the blocks (img_in, txt_norm/txt_in, the
timestep embedding, the AdaLN modulation linears, norm_out's linear and
proj_out) stay BF16 torch ops, as in the reference, where
quantize_transformer never touches them
(src/qwen_image_accel/optimizations/mxfp8.py:66-91). The modulation of all
blocks is one stacked GEMM per step.

Profiles (flags of profiles.PROFILES): quantized -> MXFP8 block GEMMs, else
BF16 torch linears; sage -> the tcgen05 Sage attention, else torch SDPA.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .kernels.attention import joint_qk_norm_rope
from .kernels.elementwise import residual
from .kernels.epilogue import layer_norm_scale_quantize_grouped
from .kernels.layernorm import layer_norm_scale
from .kernels.mxfp8 import quantize
from .kernels.scheduler import cfg_euler, proj_out_cfg_euler
from .optimizations.mxfp8 import (MXFP8Linear, matmul_gate_residual_grouped, matmul_gelu_quantize_grouped,
                                  matmul_grouped, skip_block_indices)
from .optimizations.sage_attention import (sage_attention_from_workspace, sage_attention_joint_quantized,
                                           sage_attention_split, sage_attention_split_quantized, sage_quantize_joint,
                                           workspace_bytes)
from .kernels.bf16 import gelu_tanh
from .profiles import get_profile


@dataclass(frozen=True)
class MMDiTConfig:
    num_layers: int = 60
    num_attention_heads: int = 24
    attention_head_dim: int = 128
    in_channels: int = 64
    out_channels: int = 16
    patch_size: int = 2
    joint_attention_dim: int = 3584
    axes_dims_rope: tuple = (16, 56, 56)
    eps: float = 1e-6

    @property
    def dim(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def ffn_dim(self) -> int:
        return 4 * self.dim


# ----------------------------------------------------------------------------- weights
def parameter_shapes(cfg: MMDiTConfig) -> dict[str, tuple]:
    """Diffusers state-dict names and shapes of QwenImageTransformer2DModel."""
    D, Fd, T, hd = cfg.dim, cfg.ffn_dim, cfg.joint_attention_dim, cfg.attention_head_dim
    s = {
        "img_in.weight": (D, cfg.in_channels), "img_in.bias": (D,),
        "txt_norm.weight": (T,),
        "txt_in.weight": (D, T), "txt_in.bias": (D,),
        "time_text_embed.timestep_embedder.linear_1.weight": (D, 256),
        "time_text_embed.timestep_embedder.linear_1.bias": (D,),
        "time_text_embed.timestep_embedder.linear_2.weight": (D, D),
        "time_text_embed.timestep_embedder.linear_2.bias": (D,),
        "norm_out.linear.weight": (2 * D, D), "norm_out.linear.bias": (2 * D,),
        "proj_out.weight": (cfg.patch_size ** 2 * cfg.out_channels, D),
        "proj_out.bias": (cfg.patch_size ** 2 * cfg.out_channels,),
    }
    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        for m in ("img_mod.1", "txt_mod.1"):
            s[p + m + ".weight"], s[p + m + ".bias"] = (6 * D, D), (6 * D,)
        for m in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out"):
            s[p + "attn." + m + ".weight"], s[p + "attn." + m + ".bias"] = (D, D), (D,)
        for m in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
            s[p + "attn." + m + ".weight"] = (hd,)
        for m in ("img_mlp", "txt_mlp"):
            s[p + m + ".net.0.proj.weight"], s[p + m + ".net.0.proj.bias"] = (Fd, D), (Fd,)
            s[p + m + ".net.2.weight"], s[p + m + ".net.2.bias"] = (D, Fd), (D,)
    return s


def init_parameter(name: str, shape: tuple, seed: int, device="cpu") -> torch.Tensor:
    """Seeded random init, reproducible per parameter name on a given device type:
    linear weights ~N(0, 0.02), biases ~N(0, 0.01), norm weights 1 + N(0, 0.1)."""
    g = torch.Generator(device=device).manual_seed((seed * 1000003 + zlib.crc32(name.encode())) % (2 ** 63))
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if "norm" in name and name.endswith(".weight") and len(shape) == 1:
        x = 1.0 + 0.1 * x
    elif name.endswith(".bias"):
        x = 0.01 * x
    else:
        x = 0.02 * x
    return x.to(torch.bfloat16)


# ----------------------------------------------------------------------------- RoPE / timestep
def _rope_params(index: torch.Tensor, dim: int, theta: float) -> torch.Tensor:
    freqs = torch.outer(index, 1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float32).div(dim)))
    return torch.polar(torch.ones_like(freqs), freqs)


def rope_tables(frame: int, height: int, width: int, txt_len: int, axes_dim=(16, 56, 56), theta=10000):
    """Complex64 RoPE tables (image [f*h*w, 64], text [txt_len, 64]) of the v1
    model's QwenEmbedRope(scale_rope=True)
    (WHL:diffusers/models/transformers/transformer_qwenimage.py:232-359):
    per-axis angles pos * theta^(-2i/dim); image frame index from 0, height and
    width centred (positions -(n - n//2) .. n//2 - 1); text positions start at
    max(height//2, width//2)."""
    pos = torch.arange(4096)
    neg = torch.arange(4096).flip(0) * -1 - 1
    pos_f = torch.cat([_rope_params(pos, d, theta) for d in axes_dim], dim=1)
    neg_f = torch.cat([_rope_params(neg, d, theta) for d in axes_dim], dim=1)
    split = [d // 2 for d in axes_dim]
    fp, fn = pos_f.split(split, dim=1), neg_f.split(split, dim=1)
    f_frame = fp[0][0:frame].view(frame, 1, 1, -1).expand(frame, height, width, -1)
    f_h = torch.cat([fn[1][-(height - height // 2):], fp[1][: height // 2]], 0).view(1, height, 1, -1)
    f_w = torch.cat([fn[2][-(width - width // 2):], fp[2][: width // 2]], 0).view(1, 1, width, -1)
    img = torch.cat([f_frame, f_h.expand(frame, height, width, -1), f_w.expand(frame, height, width, -1)],
                    dim=-1).reshape(frame * height * width, -1)
    start = max(height // 2, width // 2)
    txt = pos_f[start: start + txt_len]
    return img.contiguous(), txt.contiguous()


def timestep_projection(timesteps: torch.Tensor, dim: int = 256) -> torch.Tensor:
    """Sinusoidal projection of QwenTimestepProjEmbeddings.time_proj
    (flip_sin_to_cos, shift 0, scale 1000; WHL:diffusers/models/embeddings.py:27-78)."""
    half = dim // 2
    exponent = -math.log(10000) * torch.arange(0, half, dtype=torch.float32, device=timesteps.device) / half
    emb = timesteps[:, None].float() * torch.exp(exponent)[None, :]
    emb = 1000 * emb
    emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
    return torch.cat([emb[:, half:], emb[:, :half]], dim=-1)


def rms_norm_eager(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    var = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    return (x * torch.rsqrt(var + eps)).to(w.dtype) * w


# ----------------------------------------------------------------------------- model
class _LNParams:
    """Stand-in for nn.LayerNorm(dim, elementwise_affine=False, eps)."""

    def __init__(self, dim, eps):
        self.normalized_shape = (dim,)
        self.eps = eps
        self.elementwise_affine = False


class _Linear:
    """A block linear: MXFP8 (tcgen05 GEMM) when quantized, else BF16 torch."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor, quantized: bool):
        self.quantized = quantized
        self.out_features, self.in_features = w.shape
        if quantized:
            lin = torch.nn.Linear(self.in_features, self.out_features, bias=True, device=w.device, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(w)
                lin.bias.copy_(b)
            self.mx = MXFP8Linear(lin)
        else:
            self.w, self.b = w.contiguous(), b.contiguous()


class DualStreamBlock:
    def __init__(self, params: dict, prefix: str, cfg: MMDiTConfig, quantized: bool, device):
        self.quantized = quantized    # MXFP8 linears; False: bf16 (a skip block of the MXFP8 profiles)
        P = lambda n: params[prefix + n].to(device)  # noqa: E731
        cat = lambda names, suffix: torch.cat([P(f"attn.{n}.{suffix}") for n in names])  # noqa: E731
        self.img_qkv = _Linear(cat(("to_q", "to_k", "to_v"), "weight"), cat(("to_q", "to_k", "to_v"), "bias"), quantized)
        self.txt_qkv = _Linear(cat(("add_q_proj", "add_k_proj", "add_v_proj"), "weight"),
                               cat(("add_q_proj", "add_k_proj", "add_v_proj"), "bias"), quantized)
        self.img_out = _Linear(P("attn.to_out.0.weight"), P("attn.to_out.0.bias"), quantized)
        self.txt_out = _Linear(P("attn.to_add_out.weight"), P("attn.to_add_out.bias"), quantized)
        self.img_up = _Linear(P("img_mlp.net.0.proj.weight"), P("img_mlp.net.0.proj.bias"), quantized)
        self.img_down = _Linear(P("img_mlp.net.2.weight"), P("img_mlp.net.2.bias"), quantized)
        self.txt_up = _Linear(P("txt_mlp.net.0.proj.weight"), P("txt_mlp.net.0.proj.bias"), quantized)
        self.txt_down = _Linear(P("txt_mlp.net.2.weight"), P("txt_mlp.net.2.bias"), quantized)
        self.norm_q, self.norm_k = P("attn.norm_q.weight").contiguous(), P("attn.norm_k.weight").contiguous()
        self.norm_added_q = P("attn.norm_added_q.weight").contiguous()
        self.norm_added_k = P("attn.norm_added_k.weight").contiguous()


class MMDiT:
    """Qwen-Image v1 dual-stream MMDiT on the libqia_b200 kernels."""

    def __init__(self, cfg: MMDiTConfig, params, device="cuda", profile: str = "mxfp8_sage", skip_blocks=None):
        """skip_blocks: blocks whose linears stay bf16 in the MXFP8 profiles
        (default: QW21_MXFP8_SKIP_BLOCKS, else the profile's list, else
        "0,31", as the reference's quantize_transformer applies it)."""
        self.cfg, self.device = cfg, torch.device(device)
        prof = get_profile(profile)
        if not prof.fused:
            raise ValueError(f"profile {profile!r} has no fused path")
        self.quantized, self.sage = prof.quantized, prof.sage
        self.skip_blocks = skip_block_indices(skip_blocks, prof.skip_blocks) if prof.quantized else set()
        self._peer_exchanges: dict = {}
        get = params if callable(params) else (lambda n: params[n])
        dev = self.device
        G = lambda n: get(n).to(dev)  # noqa: E731
        self.img_in = (G("img_in.weight"), G("img_in.bias"))
        self.txt_norm_w = G("txt_norm.weight")
        self.txt_in = (G("txt_in.weight"), G("txt_in.bias"))
        te = "time_text_embed.timestep_embedder."
        self.t1 = (G(te + "linear_1.weight"), G(te + "linear_1.bias"))
        self.t2 = (G(te + "linear_2.weight"), G(te + "linear_2.bias"))
        self.norm_out = (G("norm_out.linear.weight"), G("norm_out.linear.bias"))
        self.proj_out = (G("proj_out.weight"), G("proj_out.bias"))
        self.blocks = []
        mod_w, mod_b = [], []
        for i in range(cfg.num_layers):
            pre = f"transformer_blocks.{i}."
            names = [pre + n for n in parameter_shapes_block_names()]
            local = {n: get(n) for n in names}
            self.blocks.append(DualStreamBlock(local, pre, cfg, self.quantized and i not in self.skip_blocks, dev))
            for m in ("img_mod.1", "txt_mod.1"):
                mod_w.append(local[pre + m + ".weight"].to(dev))
                mod_b.append(local[pre + m + ".bias"].to(dev))
            del local
        # the AdaLN modulation of every block: one [L*2*6D, D] GEMM per step
        self.mod_w = torch.cat(mod_w).contiguous()
        self.mod_b = torch.cat(mod_b).contiguous()
        del mod_w, mod_b
        self.ln = _LNParams(cfg.dim, cfg.eps)
        self._rope_cache = {}
        self._mod_stream = None

    # ------------------------------------------------------------------ helpers
    def rope(self, img_shape, txt_len):
        key = (tuple(img_shape), txt_len)
        if key not in self._rope_cache:
            img, txt = rope_tables(*img_shape, txt_len, self.cfg.axes_dims_rope)
            self._rope_cache[key] = (torch.view_as_real(img).to(self.device).contiguous(),
                                     torch.view_as_real(txt).to(self.device).contiguous())
        return self._rope_cache[key]

    def time_embed(self, timestep: torch.Tensor) -> torch.Tensor:
        proj = timestep_projection(timestep).to(torch.bfloat16)
        h = F.silu(F.linear(proj, *self.t1))
        return F.linear(h, *self.t2)

    def _linear(self, lin: _Linear, x2d: torch.Tensor) -> torch.Tensor:
        if lin.quantized:
            return lin.mx.matmul(quantize(x2d))
        return F.linear(x2d, lin.w, lin.b)

    def _attention(self, q, k, v, split, out_txt, out_img):
        if self.sage:
            sage_attention_split(q, k, v, split, out_txt, out_img, workspace=self._attn_ws(q, k))
        else:
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
            out_txt.copy_(o[:, :split])
            out_img.copy_(o[:, split:])

    def _peer_exchange(self, plan, s_loc: int, txt_len: int):
        """The PeerExchange of this plan's Ulysses group for these sizes,
        built on first use by every rank of the group together (outside CUDA
        graph capture: the first step runs eagerly)."""
        from .ulysses import PeerExchange
        key = (id(plan.group), s_loc, txt_len)
        px = self._peer_exchanges.get(key)
        if px is None:
            px = self._peer_exchanges[key] = PeerExchange(plan, s_loc, txt_len, self.cfg.num_attention_heads,
                                                          self.device)
        return px

    def _attn_ws(self, q, k):
        need = workspace_bytes(q.shape[0], q.shape[2], q.shape[1], k.shape[1])
        return torch.empty(need, device=q.device, dtype=torch.uint8)

    def _attn_ws_joint(self, batch, seq):
        need = workspace_bytes(batch, self.cfg.num_attention_heads, seq, seq)
        return torch.empty(need, device=self.device, dtype=torch.uint8)

    # ------------------------------------------------------------------ block
    def block_forward(self, blk: DualStreamBlock, x: torch.Tensor, c: torch.Tensor, mod_img, mod_txt,
                      freqs_img, freqs_txt):
        """x: image stream [B, Li, D] (updated in place), c: text stream [B, Lt, D].
        mod_*: the six (B, 1, D) modulation vectors (shift1, 1+scale1, gate1,
        shift2, 1+scale2, gate2)."""
        cfg = self.cfg
        B, Li, D = x.shape
        Lt = c.shape[1]
        H, hd = cfg.num_attention_heads, cfg.attention_head_dim
        sh1_i, s1_i, g1_i, sh2_i, s2_i, g2_i = mod_img
        sh1_t, s1_t, g1_t, sh2_t, s2_t, g2_t = mod_txt
        # ---- norm1 + modulation + Q|K|V projections
        mx = blk.quantized
        if mx:
            # image and text projections share N and K: one grouped launch
            a_i, a_t = layer_norm_scale_quantize_grouped([(x, s1_i, sh1_i), (c, s1_t, sh1_t)], self.ln)
            qkv_i, qkv_t = matmul_grouped([(blk.img_qkv.mx, a_i), (blk.txt_qkv.mx, a_t)])
            del a_i, a_t
        else:
            qkv_i = F.linear(layer_norm_scale(x, s1_i, self.ln, shift=sh1_i), blk.img_qkv.w, blk.img_qkv.b)
            qkv_t = F.linear(layer_norm_scale(c, s1_t, self.ln, shift=sh1_t), blk.txt_qkv.w, blk.txt_qkv.b)
        S = Lt + Li
        if mx and self.sage:
            # ---- QK-RMSNorm + RoPE + Sage quantization straight from the two
            # projections, joint attention, per-stream MXFP8 outputs for the
            # output projections (no bf16 Q/K/V or attention output in memory)
            qa_t, qa_i = sage_attention_joint_quantized(
                qkv_t.view(B, Lt, 3 * D), qkv_i.view(B, Li, 3 * D), (blk.norm_added_q, blk.norm_added_k),
                (blk.norm_q, blk.norm_k), freqs_txt, freqs_img, H, cfg.eps, workspace=self._attn_ws_joint(B, S))
            del qkv_t, qkv_i
            matmul_gate_residual_grouped([(blk.img_out.mx, qa_i, g1_i, x), (blk.txt_out.mx, qa_t, g1_t, c)])
            del qa_t, qa_i
        else:
            # ---- QK-RMSNorm + RoPE into the joint [text, image] sequence
            q = torch.empty(B, S, H, hd, device=x.device, dtype=torch.bfloat16)
            k = torch.empty_like(q)
            v = torch.empty_like(q)
            joint_qk_norm_rope(qkv_t.view(B, Lt, 3 * D), blk.norm_added_q, blk.norm_added_k, freqs_txt, q, k, v, 0,
                               cfg.eps)
            joint_qk_norm_rope(qkv_i.view(B, Li, 3 * D), blk.norm_q, blk.norm_k, freqs_img, q, k, v, Lt, cfg.eps)
            # ---- joint attention, written back per stream
            a_t = torch.empty(B, Lt, H, hd, device=x.device, dtype=torch.bfloat16)
            a_i = torch.empty(B, Li, H, hd, device=x.device, dtype=torch.bfloat16)
            self._attention(q, k, v, Lt, a_t, a_i)
            del q, k, v
        # ---- output projections + gated residual (in place on the streams)
        if mx and self.sage:
            pass
        elif mx:
            matmul_gate_residual_grouped([(blk.img_out.mx, quantize(a_i.view(B * Li, D)), g1_i, x),
                                          (blk.txt_out.mx, quantize(a_t.view(B * Lt, D)), g1_t, c)])
        else:
            x = residual(x, F.linear(a_i.view(B, Li, D), blk.img_out.w, blk.img_out.b), g1_i)
            c = residual(c, F.linear(a_t.view(B, Lt, D), blk.txt_out.w, blk.txt_out.b), g1_t)
        # ---- norm2 + modulation + GELU-tanh MLP + gated residual
        if mx:
            n_i, n_t = layer_norm_scale_quantize_grouped([(x, s2_i, sh2_i), (c, s2_t, sh2_t)], self.ln)
            hi, ht = matmul_gelu_quantize_grouped([(blk.img_up.mx, n_i), (blk.txt_up.mx, n_t)])
            del n_i, n_t
            matmul_gate_residual_grouped([(blk.img_down.mx, hi, g2_i, x), (blk.txt_down.mx, ht, g2_t, c)])
        else:
            hi = gelu_tanh(F.linear(layer_norm_scale(x, s2_i, self.ln, shift=sh2_i), blk.img_up.w, blk.img_up.b))
            x = residual(x, F.linear(hi, blk.img_down.w, blk.img_down.b), g2_i)
            ht = gelu_tanh(F.linear(layer_norm_scale(c, s2_t, self.ln, shift=sh2_t), blk.txt_up.w, blk.txt_up.b))
            c = residual(c, F.linear(ht, blk.txt_down.w, blk.txt_down.b), g2_t)
        return x, c

    # ------------------------------------------------------------------ sharded block
    def block_forward_sharded(self, blk: DualStreamBlock, x: torch.Tensor, c: torch.Tensor, mod_img, mod_txt,
                              freqs_img, freqs_txt, plan):
        """block_forward for one rank of a Ulysses group (see ulysses.py): x is
        this rank's image tokens [B, S_loc, D], c the replicated text stream
        [B, Lt, D], freqs_img the RoPE table of every image token of the half.
        Joint attention runs on this rank's H/U heads over every token; the
        results are the unsharded block's.

        With MXFP8 projections and Sage attention, the image tokens' q|k|v
        projection rows of this rank's heads cross before any QK-norm/RoPE, and
        the fused QK-norm + RoPE + Sage quantizer reads them (and the text rows
        of the same heads) in the projection layout: the bf16 Q/K/V never exist
        in memory, as on one GPU. With one CFG row per rank (B = 1) the rows
        of every Sage block (MXFP8 or bf16 projections) cross through NVLink
        peer memory (ulysses.PeerExchange: a scatter kernel into the heads'
        owners, and the attention kernel storing its output straight into the
        tokens' owners); otherwise, or with QIA_ULYSSES_P2P=0, through
        torch.distributed all-to-alls."""
        from .ulysses import (gather_heads, gather_heads_into, head_to_seq, head_to_seq_into, peer_exchange_enabled,
                              projection_heads, projection_to_heads, seq_to_head)
        cfg = self.cfg
        B, Sl, D = x.shape
        Lt = c.shape[1]
        H, hd = cfg.num_attention_heads, cfg.attention_head_dim
        U = plan.ulysses
        Hl, h0 = H // U, plan.u * (H // U)
        sh1_i, s1_i, g1_i, sh2_i, s2_i, g2_i = mod_img
        sh1_t, s1_t, g1_t, sh2_t, s2_t, g2_t = mod_txt
        mx = blk.quantized
        S = Lt + U * Sl
        px = self._peer_exchange(plan, Sl, Lt) if (self.sage and B == 1 and peer_exchange_enabled()) else None
        if mx:
            a_i, a_t = layer_norm_scale_quantize_grouped([(x, s1_i, sh1_i), (c, s1_t, sh1_t)], self.ln)
            qkv_i, qkv_t = matmul_grouped([(blk.img_qkv.mx, a_i), (blk.txt_qkv.mx, a_t)])
            del a_i, a_t
        else:
            qkv_i = F.linear(layer_norm_scale(x, s1_i, self.ln, shift=sh1_i), blk.img_qkv.w, blk.img_qkv.b)
            qkv_t = F.linear(layer_norm_scale(c, s1_t, self.ln, shift=sh1_t), blk.txt_qkv.w, blk.txt_qkv.b)
        if px is None:
            a_t = torch.empty(B, Lt, H, hd, device=x.device, dtype=torch.bfloat16)
            a_i = torch.empty(B, Sl, H, hd, device=x.device, dtype=torch.bfloat16)
        if px is not None:
            # NVLink peer-memory exchanges: the q|k|v rows scattered to the
            # heads' owners, the attention output stored by the attention
            # kernel into the tokens' owners
            recv = px.scatter_qkv(qkv_i.reshape(Sl, 3 * D))
            qkv_th = projection_heads(qkv_t.reshape(Lt, 3 * D), H, plan)
            ws = sage_quantize_joint(qkv_th[None], recv[None], (blk.norm_added_q, blk.norm_added_k),
                                     (blk.norm_q, blk.norm_k), freqs_txt, freqs_img, Hl, cfg.eps)
            del qkv_i, qkv_t, qkv_th
            img_out, txt_out = px.attention(ws["_workspace"])
            del ws
            a_i, a_t = img_out.view(1, Sl, H, hd), txt_out.view(1, Lt, H, hd)
        elif mx and self.sage:
            qkv_i, qkv_t = qkv_i.view(B, Sl, 3 * D), qkv_t.view(B, Lt, 3 * D)
            for b in range(B):
                qkv_ih = projection_to_heads(qkv_i[b], H, plan)       # [U * S_loc, 3 * Hl * hd]
                qkv_th = projection_heads(qkv_t[b], H, plan)          # [Lt, 3 * Hl * hd]
                ws = sage_quantize_joint(qkv_th[None], qkv_ih[None], (blk.norm_added_q, blk.norm_added_k),
                                         (blk.norm_q, blk.norm_k), freqs_txt, freqs_img, Hl, cfg.eps)
                del qkv_ih, qkv_th
                o = torch.empty(1, S, Hl, hd, device=x.device, dtype=torch.bfloat16)
                sage_attention_from_workspace(ws["_workspace"], o)
                del ws
                head_to_seq_into(o[0, Lt:], a_i[b], plan)
                gather_heads_into(o[0, :Lt], a_t[b], plan)
                del o
            del qkv_i, qkv_t
        else:
            # local Q/K/V: image tokens (all heads), text tokens (all heads)
            lo, hi = plan.image_slice(U * Sl)
            qi, ki, vi = (torch.empty(B, Sl, H, hd, device=x.device, dtype=torch.bfloat16) for _ in range(3))
            qt, kt, vt = (torch.empty(B, Lt, H, hd, device=x.device, dtype=torch.bfloat16) for _ in range(3))
            joint_qk_norm_rope(qkv_i.view(B, Sl, 3 * D), blk.norm_q, blk.norm_k, freqs_img[lo:hi].contiguous(),
                               qi, ki, vi, 0, cfg.eps)
            joint_qk_norm_rope(qkv_t.view(B, Lt, 3 * D), blk.norm_added_q, blk.norm_added_k, freqs_txt, qt, kt, vt,
                               0, cfg.eps)
            # joint [text, image] sequence of this rank's heads
            for b in range(B):
                qj, kj, vj = (torch.empty(1, S, Hl, hd, device=x.device, dtype=torch.bfloat16) for _ in range(3))
                for dst, src_t, src_i in ((qj, qt, qi), (kj, kt, ki), (vj, vt, vi)):
                    dst[0, :Lt].copy_(src_t[b, :, h0:h0 + Hl])
                    seq_to_head(src_i[b], plan, out=dst[0, Lt:])
                o_t = torch.empty(1, Lt, Hl, hd, device=x.device, dtype=torch.bfloat16)
                o_i = torch.empty(1, U * Sl, Hl, hd, device=x.device, dtype=torch.bfloat16)
                self._attention(qj, kj, vj, Lt, o_t, o_i)
                del qj, kj, vj
                a_i[b] = head_to_seq(o_i[0], plan)
                a_t[b] = gather_heads(o_t[0], plan)
            del qi, ki, vi, qt, kt, vt
        if not mx:
            x = residual(x, F.linear(a_i.view(B, Sl, D), blk.img_out.w, blk.img_out.b), g1_i)
            c = residual(c, F.linear(a_t.view(B, Lt, D), blk.txt_out.w, blk.txt_out.b), g1_t)
            hi = gelu_tanh(F.linear(layer_norm_scale(x, s2_i, self.ln, shift=sh2_i), blk.img_up.w, blk.img_up.b))
            x = residual(x, F.linear(hi, blk.img_down.w, blk.img_down.b), g2_i)
            ht = gelu_tanh(F.linear(layer_norm_scale(c, s2_t, self.ln, shift=sh2_t), blk.txt_up.w, blk.txt_up.b))
            c = residual(c, F.linear(ht, blk.txt_down.w, blk.txt_down.b), g2_t)
            return x, c
        matmul_gate_residual_grouped([(blk.img_out.mx, quantize(a_i.view(B * Sl, D)), g1_i, x),
                                      (blk.txt_out.mx, quantize(a_t.view(B * Lt, D)), g1_t, c)])
        n_i, n_t = layer_norm_scale_quantize_grouped([(x, s2_i, sh2_i), (c, s2_t, sh2_t)], self.ln)
        hi, ht = matmul_gelu_quantize_grouped([(blk.img_up.mx, n_i), (blk.txt_up.mx, n_t)])
        del n_i, n_t
        matmul_gate_residual_grouped([(blk.img_down.mx, hi, g2_i, x), (blk.txt_down.mx, ht, g2_t, c)])
        return x, c

    # ------------------------------------------------------------------ model
    def modulations(self, temb: torch.Tensor):
        """All blocks' AdaLN vectors from one stacked GEMM: per block and stream
        (shift1, 1+scale1, gate1, shift2, 1+scale2, gate2), each (B, 1, D);
        with one temb row they are (1, 1, D) views shared by every batch row."""
        D, L = self.cfg.dim, self.cfg.num_layers
        B = temb.shape[0]
        allm = F.linear(F.silu(temb), self.mod_w, self.mod_b)          # [B, L*2*6D]
        if B == 1:
            v = allm.view(L, 2, 6, D)
            v[:, :, 1] += 1          # 1 + scale1, in place over every block
            v[:, :, 4] += 1          # 1 + scale2
            return [[tuple(v[i, s, j].view(1, 1, D) for j in range(6)) for s in range(2)] for i in range(L)]
        allm = allm.view(B, L, 2, 6, D)
        out = []
        for i in range(L):
            per = []
            for s in range(2):
                m = allm[:, i, s]
                shift1, scale1, gate1 = m[:, 0:1].contiguous(), m[:, 1:2], m[:, 2:3].contiguous()
                shift2, scale2, gate2 = m[:, 3:4].contiguous(), m[:, 4:5], m[:, 5:6].contiguous()
                per.append((shift1, (1 + scale1).contiguous(), gate1, shift2, (1 + scale2).contiguous(), gate2))
            out.append(per)
        return out

    def modulations_overlapped(self, temb: torch.Tensor):
        """modulations() for a single temb row, block by block with
        qia_adaln_modulation: block 0's on the current stream (full grid),
        blocks 1.. on a side stream with one CTA per SM, so that they run
        beside the earlier blocks' kernels instead of as one weight-read-bound
        GEMV before block 0. Returns (mods, events): block i must wait for
        events[i] (None for block 0) on the stream that runs it."""
        from .kernels.modulation import adaln_modulation
        D, L = self.cfg.dim, self.cfg.num_layers
        n = 12 * D
        x = F.silu(temb).reshape(-1).contiguous()
        buf = torch.empty(L, n, device=temb.device, dtype=torch.bfloat16)
        adaln_modulation(x, self.mod_w[:n], self.mod_b[:n], D, out=buf[0])
        if self._mod_stream is None:
            self._mod_stream = torch.cuda.Stream(device=temb.device)
        side, main = self._mod_stream, torch.cuda.current_stream(temb.device)
        sms = torch.cuda.get_device_properties(temb.device).multi_processor_count
        side.wait_stream(main)
        events = [None]
        with torch.cuda.stream(side):
            for i in range(1, L):
                adaln_modulation(x, self.mod_w[i * n:(i + 1) * n], self.mod_b[i * n:(i + 1) * n], D, out=buf[i],
                                 ctas=sms)
                ev = torch.cuda.Event()
                ev.record(side)
                events.append(ev)
        # x and buf were allocated on the main stream and are read / written by
        # the side stream's launches: without these the caching allocator may
        # hand their blocks to main-stream tensors while those launches run.
        x.record_stream(side)
        buf.record_stream(side)
        v = buf.view(L, 2, 6, D)
        mods = [[tuple(v[i, s, j].view(1, 1, D) for j in range(6)) for s in range(2)] for i in range(L)]
        return mods, events

    def forward(self, hidden_states: torch.Tensor, encoder_hidden_states: torch.Tensor, timestep: torch.Tensor,
                img_shape, shared_timestep: bool = False) -> torch.Tensor:
        """hidden_states [B, Li, 64] bf16 (packed latents), encoder_hidden_states
        [B, Lt, joint_attention_dim] bf16, timestep [B] (sigma in [0, 1]);
        returns the velocity [B, Li, patch^2 * out_channels] bf16.

        shared_timestep: every batch row has the same timestep (the CFG
        batch), so the timestep embedding and modulation are computed once."""
        y = self.forward_hidden(hidden_states, encoder_hidden_states, timestep, img_shape, shared_timestep)
        return F.linear(y, *self.proj_out)

    def forward_hidden(self, hidden_states: torch.Tensor, encoder_hidden_states: torch.Tensor,
                       timestep: torch.Tensor, img_shape, shared_timestep: bool = False) -> torch.Tensor:
        """forward() up to proj_out: the norm_out output [B, Li, D] bf16."""
        cfg = self.cfg
        x = F.linear(hidden_states, *self.img_in)
        t = timestep.to(torch.bfloat16)
        c = F.linear(rms_norm_eager(encoder_hidden_states, self.txt_norm_w, cfg.eps), *self.txt_in)
        temb = self.time_embed(t[:1] if shared_timestep else t)
        freqs_img, freqs_txt = self.rope(img_shape, c.shape[1])
        if temb.shape[0] == 1:
            mods, events = self.modulations_overlapped(temb)
        else:
            mods, events = self.modulations(temb), [None] * cfg.num_layers
        x, c = x.contiguous(), c.contiguous()
        main = torch.cuda.current_stream(x.device)
        for blk, (m_img, m_txt), ev in zip(self.blocks, mods, events):
            if ev is not None:
                main.wait_event(ev)
            x, c = self.block_forward(blk, x, c, m_img, m_txt, freqs_img, freqs_txt)
        emb = F.linear(F.silu(temb), *self.norm_out)
        scale, shift = emb.chunk(2, dim=1)
        return layer_norm_scale(x, (1 + scale)[:, None].contiguous(), self.ln, shift=shift[:, None].contiguous())

    @staticmethod
    def schedule(sigma, sigma_next, device) -> torch.Tensor:
        """The step's (sigma, sigma_next) as the device float32 pair the step
        kernels read (a tensor given as `sigma` is taken as that pair)."""
        if isinstance(sigma, torch.Tensor):
            return sigma
        return torch.tensor([sigma, sigma_next], dtype=torch.float32).to(device, non_blocking=True)

    def denoise_step(self, latents: torch.Tensor, prompt_embeds: torch.Tensor, negative_embeds: torch.Tensor,
                     sigma, sigma_next, img_shape, cfg_scale: float = 4.0,
                     out: torch.Tensor | None = None) -> torch.Tensor:
        """One flow-matching Euler step with true CFG batched as B = 2
        (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
        schedulers/scheduling_flow_match_euler_discrete.py:483-517): the
        transformer on [latents, latents] with [prompt, negative] embeddings,
        then proj_out, the CFG combine and the Euler update in one kernel
        (qia_proj_out_cfg_euler). sigma, sigma_next: host floats, or `sigma`
        a device float32 tensor holding both (what a captured step reads; see
        optimizations/cuda_graph.DenoiseStepGraph). out: the updated latents'
        buffer (may be latents)."""
        b = latents.shape[0]
        sig = self.schedule(sigma, sigma_next, latents.device)
        x_in = torch.cat([latents, latents])
        enc = torch.cat([prompt_embeds, negative_embeds])
        t = sig[:1].to(latents.dtype).expand(2 * b)
        y = self.forward_hidden(x_in, enc, t, img_shape, shared_timestep=True)
        w, bias = self.proj_out
        return proj_out_cfg_euler(y, w, bias, latents.contiguous(), cfg_scale, sig, out=out)


    def forward_sharded(self, hidden_local: torch.Tensor, encoder_hidden_states: torch.Tensor,
                        timestep: torch.Tensor, img_shape, plan) -> torch.Tensor:
        """forward() for one rank of a Ulysses group: hidden_local holds this
        rank's image tokens [B, S_loc, 64] (plan.image_slice of the packed
        latents), the text and timestep are the full ones (all rows share the
        timestep); returns the velocity of this rank's tokens [B, S_loc, 64]."""
        cfg = self.cfg
        x = F.linear(hidden_local, *self.img_in)
        t = timestep.to(torch.bfloat16)
        c = F.linear(rms_norm_eager(encoder_hidden_states, self.txt_norm_w, cfg.eps), *self.txt_in)
        temb = self.time_embed(t[:1])
        freqs_img, freqs_txt = self.rope(img_shape, c.shape[1])
        lo, hi = plan.image_slice(freqs_img.shape[0])
        freqs_loc = freqs_img[lo:hi].contiguous()
        mods, events = self.modulations_overlapped(temb)
        x, c = x.contiguous(), c.contiguous()
        main = torch.cuda.current_stream(x.device)
        for blk, (m_img, m_txt), ev in zip(self.blocks, mods, events):
            if ev is not None:
                main.wait_event(ev)
            if plan.ulysses == 1:
                # CFG split only: this rank holds every token of its half, so
                # the fused single-GPU block applies unchanged
                x, c = self.block_forward(blk, x, c, m_img, m_txt, freqs_loc, freqs_txt)
            else:
                x, c = self.block_forward_sharded(blk, x, c, m_img, m_txt, freqs_img, freqs_txt, plan)
        emb = F.linear(F.silu(temb), *self.norm_out)
        scale, shift = emb.chunk(2, dim=1)
        y = layer_norm_scale(x, (1 + scale)[:, None].contiguous(), self.ln, shift=shift[:, None].contiguous())
        return F.linear(y, *self.proj_out)

    def denoise_step_sharded(self, latents_local: torch.Tensor, prompt_embeds: torch.Tensor,
                             negative_embeds: torch.Tensor, sigma: float, sigma_next: float, img_shape, plan,
                             cfg_scale: float = 4.0) -> torch.Tensor:
        """denoise_step() split over ranks: CFG half 0 runs the prompt, half 1 the
        negative prompt, each on its Ulysses group; latents_local is this rank's
        token shard [b, S_loc, 64] and the updated shard is returned."""
        from .ulysses import exchange_cfg
        if not plan.cfg_split:
            raise ValueError("denoise_step_sharded needs a plan with a CFG split")
        b = latents_local.shape[0]
        sig = self.schedule(sigma, sigma_next, latents_local.device)
        enc = prompt_embeds if plan.half == 0 else negative_embeds
        t = sig[:1].to(latents_local.dtype).expand(b)
        v = self.forward_sharded(latents_local, enc, t, img_shape, plan)
        cond, neg = exchange_cfg(v, plan)
        return cfg_euler(cond.contiguous(), neg.contiguous(), latents_local.contiguous(), cfg_scale, sigmas=sig)


def parameter_shapes_block_names() -> list[str]:
    """Relative names of one block's parameters."""
    names = []
    for m in ("img_mod.1", "txt_mod.1"):
        names += [m + ".weight", m + ".bias"]
    for m in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out"):
        names += ["attn." + m + ".weight", "attn." + m + ".bias"]
    for m in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
        names.append("attn." + m + ".weight")
    for m in ("img_mlp", "txt_mlp"):
        names += [m + ".net.0.proj.weight", m + ".net.0.proj.bias", m + ".net.2.weight", m + ".net.2.bias"]
    return names


def random_parameters(cfg: MMDiTConfig, seed: int, device="cpu"):
    """A lazy name -> tensor source of seeded random weights (see init_parameter)."""
    shapes = parameter_shapes(cfg)
    return lambda name: init_parameter(name, shapes[name], seed, device)
