"""ctypes binding of libqia_b200.so (the C ABI declared in include/qia_b200.h).

The library is loaded from this package directory. There is no fallback: if
the shared library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqia_b200.so"

_P = ctypes.c_void_p
_I = ctypes.c_int64
_F = ctypes.c_float



class GemmProblem(ctypes.Structure):
    """qia_mxfp8_gemm_problem: one GEMM of a qia_mxfp8_gemm_grouped launch."""
    _fields_ = [("a_values", _P), ("a_scales", _P), ("b_values", _P), ("b_scales", _P), ("bias", _P),
                ("gate", _P), ("resid", _P), ("out", _P), ("ldo", _I), ("q_values", _P), ("q_scales", _P),
                ("m", _I), ("rows_per_batch", _I)]


EPI_BF16, EPI_GELU_QUANT, EPI_GATE_RESIDUAL, EPI_GELU_BF16 = 0, 1, 2, 3


class LnProblem(ctypes.Structure):
    """qia_ln_mod_quant_problem: one problem of a qia_ln_mod_quant_grouped launch."""
    _fields_ = [("x", _P), ("scale", _P), ("shift", _P), ("q_values", _P), ("q_scales", _P), ("rows", _I),
                ("rows_per_batch", _I)]

# name -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "qia_mxfp8_gemm_grouped": [ctypes.c_int, _P, ctypes.c_int, _I, _I, _P],
    "qia_ln_mod_quant_grouped": [_P, ctypes.c_int, _I, _F, _P],
    "qia_adaln_modulation": [_P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qia_cfg_euler": [_P, _P, _P, _P, _I, _I, _F, _F, _P],
    "qia_cfg_euler_sched": [_P, _P, _P, _P, _I, _I, _F, _P, _P],
    "qia_rope21_table": [_P, _I, _P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P],
    "qia_proj_out_cfg_euler": [_P, _P, _P, _P, _P, _I, _I, _I, _F, _P, _P],
    "qia_ln_mod": [_P, _P, _P, _P, _I, _I, _I, _F, _P],
    "qia_ln_mod_quant": [_P, _P, _P, _P, _P, _I, _I, _I, _F, _P],
    "qia_gated_residual": [_P, _P, _P, _P, _I, _I, _I, _P],
    "qia_adaln_residual": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P],
    "qia_rms_norm": [_P, _P, _P, _I, _I, _F, _P],
    "qia_rope_qk": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qia_qknorm_rope_pack": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _F, _P],
    "qia_qknorm_rope_segment": [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _F, _P],
    "qia_swiglu": [_P, _P, _P, _I, _P],
    "qia_swiglu_quant": [_P, _P, _P, _P, _I, _I, _P],
    "qia_gelu_tanh": [_P, _P, _I, _P],
    "qia_mxfp8_quantize": [_P, _I, _P, _P, _I, _I, _P],
    "qia_mxfp8_gemm": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qia_mxfp8_gemm_gelu": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qia_mxfp8_gemm_gelu_quant": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qia_mxfp8_gemm_gate_residual": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P],
    "qia_device_error": [_P],
    "qia_sage_attention": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _F, _P, _I, _P],
    "qia_mxfp8_gemm_swiglu_quant": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "qia_sage_attention_prefill": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _F, _P, _I, _P],
    "qia_sage_attention_split": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _F, _P, _I, _P],
    "qia_sage_attention_split_mx": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _F, _P, _I, _P],
    "qia_sage_attention_noalloc": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _F, _P],
    "qia_sage_quantize": [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P],
    "qia_sage_quantize_joint": [_P, _I, _P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P],
    "qia_sage_attention_joint_mx": [_P, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                                    _F, _F, _P, _I, _P],
    "qia_sage_attn_quantized": [_P, _P, _I, _I, _I, _I, _I, _P, _F, _P],
}

SIGNATURES.update({
    "qia_ipc_alloc": [_I, ctypes.POINTER(ctypes.c_void_p), _P],
    "qia_ipc_open": [_P, ctypes.POINTER(ctypes.c_void_p)],
    "qia_ipc_close": [_P],
    "qia_ipc_free": [_P],
    "qia_ulysses_scatter_qkv": [_P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P],
    "qia_ulysses_wait": [_P, _P, _I, _I, _I, _P],
    "qia_sage_attn_quantized_peers": [_P, _I, _I, _I, _I, _P, _P, _I, _I, _I, _I, _P, _I, _F, _P],
})

# entry points that do not return a status code: name -> (restype, argtypes)
RAW_SIGNATURES: dict[str, tuple] = {
    "qia_sage_workspace_bytes": (ctypes.c_int64, [_I, _I, _I, _I]),
    "qia_ipc_handle_bytes": (ctypes.c_int64, []),
    "qia_sage_attn_ctas": (ctypes.c_int64, [_I, _I, _I]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class QiaError(RuntimeError):
    """A qia_* entry point returned a non-zero status."""

    def __init__(self, name: str, code: int, message: str):
        super().__init__(f"{name} failed with status {code}: {message}")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                                   "`python qwen-image-2.1-accel_b200/build.py` (no CPU fallback exists)")
            lib = ctypes.CDLL(str(LIB_PATH))
            lib.qia_last_error_string.restype = ctypes.c_char_p
            lib.qia_last_error_string.argtypes = []
            lib.qia_abi_version.restype = ctypes.c_int
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            for name, (res, args) in RAW_SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def declared_symbols() -> list[str]:
    return ["qia_last_error_string", "qia_abi_version", *SIGNATURES, *RAW_SIGNATURES]


# kernels each entry point queues (for launch accounting); default 1
KERNELS_PER_CALL = {"qia_sage_attention": 4, "qia_sage_attention_split": 4, "qia_sage_quantize": 3,
                    "qia_sage_attention_split_mx": 4, "qia_sage_quantize_joint": 3, "qia_sage_attention_joint_mx": 4,
                    "qia_sage_attention_noalloc": 4, "qia_sage_attention_prefill": 4,
                    "qia_device_error": 0}
launch_count = 0


def call(name: str, *args) -> None:
    """Invoke a qia_* entry point and raise QiaError on a non-zero status."""
    global launch_count
    lib = load()
    launch_count += KERNELS_PER_CALL.get(name, 1)
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.qia_last_error_string().decode(errors="replace")
        raise QiaError(name, rc, msg)


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the device)."""
    v = ctypes.c_int(0)
    call("qia_device_error", ctypes.byref(v))
    return v.value


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device: torch.device | None = None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("qwen_image_accel_b200 ops run on CUDA tensors only (no CPU path)")
