"""The MXFP8 / Sage profiles' decode installer on the sm_100a kernels.

Same name and contract as the reference's src/qwen_image_accel/optimizations/
quantized_decode.py:108-137 (`install_mx_fused_decode(transformer, sage)`,
with the `MXFusedProcessor` attention processor, :31-78): on a Diffusers
Qwen-Image 2.1 transformer whose block linears quantize_transformer has made
MXFP8, the cached decode steps run one LayerNorm -> MXFP8 per consumer group,
the stacked Q|K|V MXFP8 GEMM, the fused QK-RMSNorm + RoPE + prefix pack, the
tcgen05 Sage attention when `sage` and nothing is masked (its output quantized
to MXFP8 in the attention epilogue), and the output / down projections with
the gated residual in the GEMM epilogue; the MLP's gate and value projections
share one quantized activation and the SwiGLU is fused with the quantization
of the down projection's operand. Blocks left in bf16 (skip_blocks) take the
same fused path with bf16 GEMMs. The prefill keeps the native forward (with
the MXFP8 linears and this MLP). See optimizations/decode.py for the routing.
"""
from __future__ import annotations

from .decode import processor_class, route_blocks


def MXFusedProcessor(sage: bool = False):  # noqa: N802  (a class factory: Diffusers is imported on first use)
    """A Diffusers attention processor whose cached-decode calls run the
    MXFP8/fused projections, pack and (with sage, when unmasked) the Sage
    attention; other calls are Diffusers'."""
    return processor_class("MXFusedProcessor")(sage=sage)


def install_mx_fused_decode(transformer, sage: bool = False) -> None:
    """Route every block's cached decode through the MXFP8 (+ Sage) path."""
    route_blocks(transformer, sage=sage)
    for block in transformer.transformer_blocks:
        block.attn.set_processor(MXFusedProcessor(sage=sage))
