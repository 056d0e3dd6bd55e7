"""Supported profiles, with the reference's names and flags.

Mirrors src/qwen_image_accel/profiles.py: the same PROFILES mapping, Profile
fields and retired-name errors, so callers select the same behaviour by name.
The profile names, flags and retired-name table are the reference's interface
(Qwen-Image-2.1-Accel, Copyright (c) 2026 Devin Lai, CPAL-1.0; see its LICENSE
and NOTICE for the attribution terms); the module here is written anew.
"""
from dataclasses import dataclass
from types import MappingProxyType


@dataclass(frozen=True)
class Profile:
    description: str
    fused: bool = False
    quantized: bool = False
    sage: bool = False
    compile: bool = False
    graph: bool = False
    skip_blocks: str | None = None


PROFILES = MappingProxyType({
    "baseline": Profile("Original BF16 initialization"),
    "safe": Profile("Conservative encoder and modulation improvements"),
    "fused": Profile("Default: selective BF16 fusion", fused=True),
    "fused_sage": Profile("BF16 fusion with Sage-style INT8/FP8 attention", fused=True, sage=True),
    "mxfp8": Profile("Block-scaled FP8 linears", fused=True, quantized=True),
    "mxfp8_sage": Profile("Block-scaled FP8 with Sage-style INT8/FP8 attention", fused=True, quantized=True,
                          sage=True),
    "mxfp8_balanced": Profile("MXFP8 with six BF16 boundary blocks", fused=True,
                              quantized=True, skip_blocks="0,1,2,29,30,31"),
    "mxfp8_balanced_sage": Profile("Balanced MXFP8 with Sage-style attention", fused=True,
                                   quantized=True, sage=True, skip_blocks="0,1,2,29,30,31"),
    "compiled": Profile("Experimental bounded block compilation", compile=True),
    "graph": Profile("CUDA Graph replay of the whole denoise step", fused=True, graph=True),
})

_REMOVED = {
    "fp8": "mxfp8", "fp8_sage": "mxfp8_sage",
    "fp8_sage_compiled": "mxfp8_sage", "sage": "fused_sage",
    "fused_cudnn": "fused with QW21_ATTENTION=_native_cudnn",
    "mxfp8_cudnn": "mxfp8 with QW21_ATTENTION=_native_cudnn",
}


def get_profile(name: str) -> Profile:
    """Resolve a profile before loading weights or changing a pipeline."""
    if name in _REMOVED:
        raise ValueError(f"Profile {name!r} was retired; use {_REMOVED[name]}.")
    try:
        return PROFILES[name]
    except KeyError:
        raise ValueError(f"Unknown Qwen optimization profile {name!r}; choose {', '.join(PROFILES)}") from None
