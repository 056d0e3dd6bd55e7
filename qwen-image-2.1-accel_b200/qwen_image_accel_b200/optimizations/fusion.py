"""The `fused` profile's decode installer on the sm_100a kernels.

Same name and contract as the reference's src/qwen_image_accel/optimizations/
fusion.py:38-60 (`install_fused_decode(transformer)`, with the
`FusedRopeProcessor` attention processor): on a Diffusers Qwen-Image 2.1
transformer with bf16 linears, the cached decode steps of every block run the
fused bf16 ops (LayerNorm x (1 + scale), QK-RMSNorm + RoPE + prefix K/V pack,
gated residuals, SwiGLU) while the GEMMs stay bf16 torch linears and the
attention stays SDPA; the prefill keeps the native forward. See
optimizations/decode.py for the routing.
"""
from __future__ import annotations

from .decode import processor_class, route_blocks


def FusedRopeProcessor():  # noqa: N802  (a class factory: Diffusers is imported on first use)
    """A Diffusers attention processor whose cached-decode calls run the fused
    QK-RMSNorm + RoPE + prefix pack and SDPA; other calls are Diffusers'."""
    return processor_class("FusedRopeProcessor")(sage=False)


def install_fused_decode(transformer) -> None:
    """Route every block's cached decode through the fused bf16 path."""
    route_blocks(transformer, sage=False)
    for block in transformer.transformer_blocks:
        block.attn.set_processor(FusedRopeProcessor())
