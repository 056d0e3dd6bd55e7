"""The reference's `mxfp8_sage` composition on the Diffusers Qwen-Image (v1)
MMDiT, on the GPU -- TEST INFRASTRUCTURE, never the product.

BASELINE configs 4-5 name the v1 dual-stream MMDiT, which the reference
package never patches; its `mxfp8_sage` profile applied to that model means:

* the Diffusers QwenImageTransformer2DModel from the pinned wheel
  (WHL:diffusers/models/transformers/transformer_qwenimage.py:633-1031),
  eager bf16, for everything outside the substitutions below;
* every block linear outside the skip blocks (default "0,31",
  src/qwen_image_accel/pipeline.py:133) replaced by the reference's
  MXFP8Linear (src/qwen_image_accel/optimizations/mxfp8.py:19-41):
  activation and weight quantized by the reference's MXFP8 rule
  (kernels/mxfp8.py:31-67, restated in torch below as its known-answer test
  does, tests/gpu/check_mxfp8.py:20-34) and multiplied by torch._scaled_mm
  (cuBLASLt); the v1 linears' biases, which the reference's MXFP8Linear
  lacks, added after in bf16;
* the unmasked joint attention through the reference's SageAttention, built
  from its pinned sources (oracle/sage_ref.py);
* the pipeline's true-CFG combine with norm rescale and the flow-match Euler
  step (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
  schedulers/scheduling_flow_match_euler_discrete.py:483-517).

Weights come from the package's seeded recipe (mmdit.init_parameter), so the
same seed gives the same model as qwen_image_accel_b200.mmdit.MMDiT.
"""
from __future__ import annotations

import torch
from torch import nn

from . import diffusers_ref, sage_ref


def mx_quantize_torch(x: torch.Tensor):
    """The reference's MXFP8 quantization of a bf16 [M, K] tensor (K % 128 == 0)
    in torch ops: per 1x32 block, exponent e = the block maximum's binade - 8
    (+1 above mantissa 1.75), codes = x * 2^(127 - e) cast to E4M3, rows padded
    to 128; scales E8M0 in the 128x4 blocked layout."""
    m, k = x.shape
    mp = (m + 127) // 128 * 128
    xf = torch.zeros(mp, k, dtype=torch.float32, device=x.device)
    xf[:m] = x.float()
    blocks = xf.view(mp, k // 32, 32)
    amax = blocks.abs().amax(-1)
    bits = amax.view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 8 + ((bits & 0x7FFFFF) > 6291456).int()
    e = torch.where(amax == 0, torch.zeros_like(e), e.clamp(0, 254))
    inv = ((254 - e) << 23).view(torch.float32)
    q = (blocks * inv[..., None]).view(mp, k).to(torch.float8_e4m3fn)
    s = e.to(torch.uint8).view(mp // 128, 4, 32, k // 128, 4).permute(0, 3, 2, 1, 4).contiguous().view(-1)
    return q, s.view(torch.float8_e8m0fnu)


class ScaledMMLinear(nn.Module):
    """The reference's MXFP8Linear on a Diffusers linear (see module docstring)."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.wq, self.ws = mx_quantize_torch(lin.weight.detach().to(torch.bfloat16).contiguous())
        self.bias = None if lin.bias is None else lin.bias.detach().to(torch.bfloat16)

    def forward(self, x):
        flat = x.reshape(-1, self.in_features).contiguous()
        a, s = mx_quantize_torch(flat)
        y = torch._scaled_mm(a, self.wq.t(), scale_a=s, scale_b=self.ws, out_dtype=torch.bfloat16)[: flat.shape[0]]
        if self.bias is not None:
            y = y + self.bias
        return y.view(*x.shape[:-1], self.out_features)


_BLOCK_LINEARS = ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "attn.add_q_proj", "attn.add_k_proj",
                  "attn.add_v_proj", "attn.to_add_out", "img_mlp.net.0.proj", "img_mlp.net.2",
                  "txt_mlp.net.0.proj", "txt_mlp.net.2")


def build(num_layers: int, seed: int, device="cuda", heads: int = 24, text_dim: int = 3584,
          quantized: bool = True, sage: bool = True, skip=(0, 31)):
    """The Diffusers v1 model at the BASELINE dims (3072 hidden, heads x 128)
    with `num_layers` blocks, seeded weights, and the reference's mxfp8_sage
    substitutions (see the module docstring)."""
    from qwen_image_accel_b200.mmdit import MMDiTConfig, init_parameter, parameter_shapes
    tq = diffusers_ref.qwen_v1()
    model = tq.QwenImageTransformer2DModel(patch_size=2, in_channels=64, out_channels=16, num_layers=num_layers,
                                           attention_head_dim=128, num_attention_heads=heads,
                                           joint_attention_dim=text_dim, axes_dims_rope=(16, 56, 56))
    model = model.to(torch.bfloat16)
    shapes = parameter_shapes(MMDiTConfig(num_layers=num_layers, num_attention_heads=heads,
                                          joint_attention_dim=text_dim))
    model.load_state_dict({n: init_parameter(n, shapes[n], seed) for n in model.state_dict()})
    model = model.to(device).eval()
    if quantized:
        for i, block in enumerate(model.transformer_blocks):
            if i in skip:
                continue
            for name in _BLOCK_LINEARS:
                parent_name, _, leaf = name.rpartition(".")
                parent = block.get_submodule(parent_name)
                setattr(parent, leaf, ScaledMMLinear(getattr(parent, leaf)))
    if sage:
        native = tq.dispatch_attention_fn

        def dispatch(query, key, value, attn_mask=None, **kwargs):
            if attn_mask is None:
                return sage_ref.attention(query, key, value)
            return native(query, key, value, attn_mask=attn_mask, **kwargs)

        tq.dispatch_attention_fn = dispatch
        model._qia_restore = lambda: setattr(tq, "dispatch_attention_fn", native)
    return model


def denoise(model, latents, prompt_embeds, negative_embeds, sigmas, img_shape, cfg_scale: float = 4.0):
    """len(sigmas) - 1 Euler steps of the pipeline's true-CFG loop (the two CFG
    branches batched as B = 2, which is the same per-row arithmetic), each
    with the timestep bf16(sigma) the MMDiT receives."""
    b = latents.shape[0]
    enc = torch.cat([prompt_embeds, negative_embeds])
    sig = torch.tensor(sigmas, dtype=torch.float32)
    with torch.no_grad():
        for i in range(len(sigmas) - 1):
            t = torch.full((2 * b,), float(sigmas[i]), device=latents.device, dtype=torch.bfloat16)
            v = model(hidden_states=torch.cat([latents, latents]), encoder_hidden_states=enc, timestep=t,
                      img_shapes=[img_shape] * (2 * b), return_dict=False)[0]
            cond, neg = v[:b], v[b:]
            comb = neg + cfg_scale * (cond - neg)
            noise = comb * (torch.norm(cond, dim=-1, keepdim=True) / torch.norm(comb, dim=-1, keepdim=True))
            dt = (sig[i + 1] - sig[i]).to(latents.device)
            latents = (latents.to(torch.float32) + dt * noise).to(noise.dtype)
    return latents
