"""Cached decode of a Diffusers Qwen-Image 2.1 transformer on the sm_100a kernels.

The installers configure_pipeline calls (`install_fused_decode`,
optimizations/fusion.py; `install_mx_fused_decode`,
optimizations/quantized_decode.py) take a Diffusers
`QwenImage21Transformer2DModel` (WHL:diffusers/models/transformers/
transformer_qwenimage21.py:740-1018) and route the decode steps of its blocks
(`kv_cache_mode="cached"`: target-image tokens only, attending to the cached
prefix K/V) through `qwen21.Block21` bound to the block's own modules:

* the block's to_q / to_k / to_v are restacked into one [W_q; W_k; W_v]
  linear whose storage the three modules then share (views), so the decode
  runs one projection GEMM and the prefill still sees three linears;
* each block's forward, in cached mode, becomes Block21.forward_cached (LN x
  (1 + scale) -> MXFP8 when the projections are MXFP8, the fused QK-RMSNorm +
  RoPE + prefix pack, the tcgen05 Sage attention when the profile has it and
  nothing is masked, gate-residual epilogues, the SwiGLU MLP); every other
  mode keeps the block's own forward (the native prefill, as the reference
  keeps it: src/qwen_image_accel/optimizations/fusion.py:16-18);
* the MLP's forward becomes Block21's SwiGLU MLP in every mode (gate and
  value projections sharing one activation, SwiGLU on the kernels), as the
  reference replaces it (quantized_decode.py:141-156, kernels/bf16.py:39-43).

The per-step modulation vectors (1 + s1, tanh g1, 1 + s2, tanh g2) are
computed once per modulation tensor and shared by all blocks.
"""
from __future__ import annotations

import types

import torch

from ..qwen21 import Block21, Block21Config, modulation_values
from .mxfp8 import stack_linears

_STATE = "_qia_decode"


def _eps(module, default=1e-6):
    return float(getattr(module, "eps", default))


def bind_block(block, sage: bool) -> Block21:
    """Block21 over a Diffusers QwenImage21TransformerBlock's modules (shared
    weights; to_q/to_k/to_v restacked in place when they are all MXFP8 or all
    bf16 without bias)."""
    attn, mlp = block.attn, block.img_mlp
    dim = attn.to_q.in_features
    heads = attn.heads
    head_dim = attn.to_q.out_features // heads
    eps = _eps(block.img_norm1)
    if head_dim != 128:
        raise NotImplementedError(f"the fused decode needs head_dim 128, got {head_dim}")
    if _eps(attn.norm_q) != eps or _eps(attn.norm_k) != eps:
        raise NotImplementedError("the fused decode needs one eps for the LayerNorms and the Q/K RMSNorms")
    parts = (attn.to_q, attn.to_k, attn.to_v)
    try:
        qkv = stack_linears(parts)
    except ValueError:
        qkv = parts                     # a mixed selection: three projections, concatenated
    cfg = Block21Config(dim=dim, heads=heads, head_dim=head_dim,
                        mlp_ratio=max(1, mlp.gate_layer.out_features // dim), eps=eps)
    weight = lambda norm: norm.weight.detach().to(torch.bfloat16).contiguous()  # noqa: E731
    return Block21.bind(qkv, attn.to_out[0], (mlp.gate_layer, mlp.proj, mlp.out), weight(attn.norm_q),
                        weight(attn.norm_k), cfg, sage=sage)


def _key_valid(mask):
    """The model's decode padding mask (joint key-valid [B, 1, 1, S] bool, or
    None) as Block21's key_valid [B, S]."""
    if mask is None:
        return None
    if mask.dtype != torch.bool:
        raise NotImplementedError("the fused decode takes a boolean key-padding mask")
    return mask.reshape(mask.shape[0], -1)


def step_values(transformer, modulation: torch.Tensor):
    """modulation_values of the shared modulation [B + 1, 4D], computed once
    per modulation tensor and reused by every block of the step."""
    state = getattr(transformer, _STATE)
    if state["modulation"] is not modulation:
        state["modulation"] = modulation
        state["values"] = modulation_values(modulation)
    return state["values"]


def route_blocks(transformer, sage: bool) -> list:
    """Bind every block and install the cached-decode forward and the MLP
    forward; returns the bound Block21s (kept on the transformer)."""
    if hasattr(transformer, _STATE):
        raise RuntimeError("the decode path is already installed on this transformer")
    setattr(transformer, _STATE, {"modulation": None, "values": None, "bound": []})
    bound = getattr(transformer, _STATE)["bound"]
    for block in transformer.transformer_blocks:
        b21 = bind_block(block, sage)
        bound.append(b21)
        native = block.forward

        def forward(*args, _native=native, _b21=b21, **kwargs):
            if kwargs.get("kv_cache_mode") != "cached" or args:
                return _native(*args, **kwargs)
            values = step_values(transformer, kwargs["modulation"])
            return _b21.forward_cached(kwargs["hidden_states"], values, kwargs["rotary_emb"],
                                       kwargs["layer_cache"], key_valid=_key_valid(kwargs.get("attention_mask")))

        block.forward = forward
        block.img_mlp.forward = types.MethodType(lambda mod, x, _b21=b21: _b21._mlp(x, x.shape[:-1]),
                                                 block.img_mlp)
    return bound


def bound_blocks(transformer) -> list:
    state = getattr(transformer, _STATE, None)
    if state is None:
        raise RuntimeError("install_fused_decode / install_mx_fused_decode first")
    return state["bound"]


_PROCESSOR_CLASSES: dict = {}


def processor_class(name: str):
    """A Diffusers QwenImage21AttnProcessor subclass (created on first use, so
    that importing this package needs no Diffusers) whose cached-decode calls
    run Block21.attention_cached on the attention module's own weights; every
    other call is the Diffusers processor's."""
    if name in _PROCESSOR_CLASSES:
        return _PROCESSOR_CLASSES[name]
    from diffusers.models.transformers.transformer_qwenimage21 import QwenImage21AttnProcessor

    def __init__(self, sage: bool = False):
        self.sage = sage
        self._bound = None

    def __call__(self, attn, hidden_states, attention_mask=None, rotary_emb=None, layer_cache=None,
                 kv_cache_mode=None, cache_write_slice=None, segments=None, key_valid=None):
        if kv_cache_mode != "cached" or key_valid is not None:
            return QwenImage21AttnProcessor.__call__(self, attn, hidden_states, attention_mask, rotary_emb,
                                                     layer_cache, kv_cache_mode, cache_write_slice, segments,
                                                     key_valid)
        if self._bound is None:
            eps = _eps(attn.norm_q)
            cfg = Block21Config(dim=attn.to_q.in_features, heads=attn.heads,
                                head_dim=attn.to_q.out_features // attn.heads, eps=eps)
            w = lambda norm: norm.weight.detach().to(torch.bfloat16).contiguous()  # noqa: E731
            self._bound = Block21.bind((attn.to_q, attn.to_k, attn.to_v), attn.to_out[0], (None, None, None),
                                       w(attn.norm_q), w(attn.norm_k), cfg, sage=self.sage)
        return self._bound.attention_cached(hidden_states, rotary_emb, layer_cache,
                                            key_valid=_key_valid(attention_mask))

    cls = type(name, (QwenImage21AttnProcessor,), {"__init__": __init__, "__call__": __call__,
                                                   "__doc__": processor_class.__doc__})
    _PROCESSOR_CLASSES[name] = cls
    return cls


def broadcast_decode_modulation(transformer):
    """The non-fused profiles' decode tweak (src/qwen_image_accel/pipeline.py:
    68-91 without compilation): in cached mode every row is a target row, so
    each sample's modulation row is broadcast instead of selected per token
    (the trailing t = 0 row, which belongs to the prefix, is dropped)."""
    for block in transformer.transformer_blocks:
        native = block.forward

        def forward(*args, _native=native, **kwargs):
            if kwargs.get("kv_cache_mode") == "cached":
                kwargs["modulation"] = kwargs["modulation"][:-1]
                kwargs["target_token_mask"] = None
            return _native(*args, **kwargs)

        block.forward = forward

