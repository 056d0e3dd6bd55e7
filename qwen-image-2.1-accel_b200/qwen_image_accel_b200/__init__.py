"""B200-native (sm_100a) denoising-transformer hot path of Qwen-Image-2.1-Accel.

The public surface mirrors the reference package `qwen_image_accel`: the
profile registry (PROFILES / get_profile with `fused`, `fused_sage`,
`mxfp8_sage`, ...) and the block-level ops under `kernels` and
`optimizations`. Every op calls libqia_b200.so, a C ABI of hand-written CUDA
kernels; importing this package does not load the library (the first op does).
"""
from .profiles import PROFILES, Profile, get_profile

__version__ = "0.1.0"
__all__ = ["PROFILES", "Profile", "get_profile", "library_path"]


def library_path():
    from . import _lib
    return _lib.LIB_PATH
