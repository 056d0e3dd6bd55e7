"""configure_pipeline: put a profile's sm_100a kernels on a Diffusers Qwen-Image 2.1 pipeline.

Drop-in for the reference's `configure_pipeline(pipe, profile="fused")`
(src/qwen_image_accel/pipeline.py:109-198): same profile names, the same
checks before anything is changed (unknown or retired profile, a pipeline
configured before, a non-bf16 transformer or an unvalidated runtime for the
fused profiles), the same installers in the same order, and the same
configuration dictionary keys, returned and kept as `pipe._qw_optimization`.

What changes is what the installers run: `quantize_transformer` makes MXFP8
linears for the tcgen05 block-scaled GEMM; `install_mx_fused_decode` /
`install_fused_decode` route the cached decode through optimizations/decode.py
(LayerNorm -> MXFP8, the stacked Q|K|V GEMM, QK-RMSNorm + RoPE + prefix pack,
the tcgen05 Sage attention, gate-residual GEMM epilogues, SwiGLU fused with
the next GEMM's quantization); `install_qk_norm` / `install_swiglu` give the
native prefill the RMSNorm and SwiGLU kernels; `install_cuda_graph` replays
the decode blocks from one CUDA graph.

Only the denoising transformer is in this package's scope: the text encoder
placement, the VAE tiling policy and the step cache of the reference are not
provided here (their keys report what was left as the pipeline had it), and
the `compiled` profile (bounded torch.compile) raises.
"""
from __future__ import annotations

import hashlib
import os
from pathlib import Path

import torch

from .profiles import get_profile

# sha256 of the Diffusers transformer_qwenimage21.py the installers were
# written against (the reference pins the same file: third_party/manifest.json)
VALIDATED_TRANSFORMER_SHA256 = "0eb0555e21ca93195e1fe9389113cafbf0e8822f6454c3001cebb3d21521ebd7"
_CONFIG_ATTR = "_qw_optimization"


def _check_runtime(pipe) -> None:
    """Everything the fused profiles need, checked before any change."""
    transformer = pipe.transformer
    if next(transformer.parameters()).dtype != torch.bfloat16:
        raise ValueError("the fused profiles need a bf16 transformer")
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        raise RuntimeError("the fused profiles run on sm_100 (B200) GPUs only; use the 'baseline' profile elsewhere")
    from . import _lib
    _lib.load()                      # raises when libqia_b200.so is missing
    import importlib
    module = importlib.import_module(type(transformer).__module__)
    digest = hashlib.sha256(Path(module.__file__).read_bytes()).hexdigest()
    if digest != VALIDATED_TRANSFORMER_SHA256:
        raise RuntimeError(f"{module.__file__} is not the Diffusers Qwen-Image 2.1 transformer these installers "
                           "were validated against; use the 'baseline' profile")


def _to_cuda(pipe) -> None:
    pipe.transformer.to("cuda")
    vae = getattr(pipe, "vae", None)
    if vae is not None:
        vae.to("cuda")


def _attention_backend(transformer) -> str:
    """QW21_ATTENTION, when set, names the Diffusers attention backend of the
    non-Sage attention calls ("native"/"default": Diffusers' own choice)."""
    choice = os.environ.get("QW21_ATTENTION", "").strip()
    if not choice:
        return "native"
    backend = None if choice in ("native", "default") else choice
    for block in transformer.transformer_blocks:
        block.attn.processor._attention_backend = backend
    return backend or "native"


def configure_pipeline(pipe, profile: str = "fused") -> dict:
    """Install `profile` on `pipe` (a Diffusers QwenImage21Pipeline, or any
    object with a `.transformer` holding a QwenImage21Transformer2DModel) and
    return the configuration dictionary."""
    selected = get_profile(profile)
    if hasattr(pipe, _CONFIG_ATTR):
        raise RuntimeError("configure a fresh pipeline once; a profile cannot be switched in place")
    if selected.compile:
        raise NotImplementedError("the 'compiled' profile (bounded torch.compile) is not part of the B200 build; "
                                  "use 'graph' for launch-free decode replay")
    if selected.fused:
        _check_runtime(pipe)
    transformer = pipe.transformer
    if profile == "baseline":
        _to_cuda(pipe)
        config = {"profile": "baseline", "approximate": False}
        setattr(pipe, _CONFIG_ATTR, config)
        return config
    _to_cuda(pipe)
    config = {"profile": profile, "features_only_encoder": False, "native_bf16_prefix_cache": True,
              "dit_gpu_resident": True, "text_encoder_offload": "unchanged", "approximate": False}
    if selected.quantized:
        from .optimizations.mxfp8 import quantize_transformer
        skip = os.environ.get("QW21_MXFP8_SKIP_BLOCKS", selected.skip_blocks or "0,31")
        layers = os.environ.get("QW21_MXFP8_LAYERS", "all")
        config["mxfp8_linears"] = len(quantize_transformer(transformer, skip, layers))
        config["mxfp8_skipped_blocks"] = skip
        config["mxfp8_layer_selection"] = layers
        config["approximate"] = True
    if selected.sage:
        from .optimizations import sage_attention
        sage_attention._check_settings()
        config["sage_decode"] = True
        config["sage_pv_accum"] = sage_attention.ACCUM
        config["sage_qk_gran"] = sage_attention.QK_GRAN
        config["approximate"] = True
    if selected.fused:
        from .kernels.bf16 import install_qk_norm, install_swiglu
        composed = selected.quantized or selected.sage
        if composed:
            from .optimizations.quantized_decode import install_mx_fused_decode
            install_mx_fused_decode(transformer, sage=selected.sage)
        else:
            from .optimizations.fusion import install_fused_decode
            install_fused_decode(transformer)
        install_qk_norm(transformer)
        if not composed:
            install_swiglu(transformer)
        for key in ("fused_qk_rmsnorm", "fused_swiglu", "fused_norm_rope_kv_pack",
                    "fused_native_order_layernorm_scale", "runtime_token_counts"):
            config[key] = True
        if selected.graph:
            from .optimizations.cuda_graph import install_cuda_graph
            install_cuda_graph(transformer)
    else:
        from .optimizations.decode import broadcast_decode_modulation
        broadcast_decode_modulation(transformer)
    config["attention_backend"] = _attention_backend(transformer)
    if config["attention_backend"] != "native":
        config["approximate"] = True
    config["broadcast_decode_modulation"] = True
    config["compiled_decode_blocks"] = False
    config["cuda_graph"] = selected.graph
    config["vae_tiling"] = {"policy": "provided"}
    setattr(pipe, _CONFIG_ATTR, config)
    return config
