"""Build the reference's SageAttention CUDA extension into oracle/_ref/sage/ --
TEST INFRASTRUCTURE, never the product.

The reference's quantized attention (`src/qwen_image_accel/optimizations/
sage_attention.py:19-25`) calls `sageattn_qk_int8_pv_fp8_cuda` from the
SageAttention 2.2.0 sources it pins (third_party/sources/sageattention-d1a57a5
.tar.gz, sha256 in third_party/manifest.json:20-24). This recipe compiles the
two extension modules that call path needs, from the tarball as it lies, with
the compiler flags of the tarball's own setup.py (setup.py:51-61: `-O3
--use_fast_math`, C++17, half operators enabled) for sm_100a:

* `sage_ref_fused`  <- csrc/fused/pybind.cpp + fused.cu (the Q/K INT8 and V
  FP8 quantizers, setup.py:213-219);
* `sage_ref_qattn`  <- csrc/qattn/pybind_sm89.cpp + the seven sm89_*.cu
  kernels (the mma.sync INT8 QK / FP8 PV attention, setup.py:186-201; the sm89
  kernels are the ones the reference's call path selects, and their PTX needs
  only sm_89 features, which sm_100a has).

The tarball is extracted to a temporary directory; nothing from it is copied
into this repository. The built modules land in oracle/_ref/sage/ (git-ignored,
shipped to the GPU box with the rest of the tree). `oracle/sage_ref.py` loads
them and restates the Python call sequence of core.py around them.

Usage: python oracle/build_sage_ref.py --reference <checkout>   (or QIA_REFERENCE=<checkout>)
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tarfile
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "sage"
TARBALL = "third_party/sources/sageattention-d1a57a5.tar.gz"
SHA256 = "18ce3aebd3d04511abd01ed99de603cc88d7d4df6e81edee2565984ea4214f1c"
TOPDIR = "SageAttention-d1a57a546c3d395b1ffcbeecc66d81db76f3b4b5"

# SAGE:setup.py:51-61 and :71-73 (the ABI define), arch set to sm_100a only
CXX_FLAGS = ["-O3", "-std=c++17", "-DENABLE_BF16"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
              "--use_fast_math", "--threads=4", "-diag-suppress=174"]

MODULES = {
    "sage_ref_fused": ["csrc/fused/pybind.cpp", "csrc/fused/fused.cu"],
    "sage_ref_qattn": ["csrc/qattn/pybind_sm89.cpp",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_attn_inst_buf.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f16_attn_inst_buf.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_attn.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_fuse_v_scale_fuse_v_mean_attn.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_fuse_v_scale_attn.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_fuse_v_scale_attn_inst_buf.cu",
                       "csrc/qattn/sm89_qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf.cu"],
}


def built() -> bool:
    return all((OUT / name / f"{name}.so").exists() for name in MODULES)


def build(reference: Path, force: bool = False, verbose: bool = False) -> Path:
    tar = reference / TARBALL
    digest = hashlib.sha256(tar.read_bytes()).hexdigest()
    if digest != SHA256:
        raise RuntimeError(f"{tar}: sha256 {digest} does not match the pinned {SHA256}")
    if built() and not force:
        return OUT
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(max(1, min(8, os.cpu_count() or 1))))
    import torch
    from torch.utils import cpp_extension
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    with tempfile.TemporaryDirectory(prefix="qia_sage_src_") as tmp:
        with tarfile.open(tar) as tf:
            tf.extractall(tmp, filter="data")
        src = Path(tmp) / TOPDIR
        for name, files in MODULES.items():
            bdir = OUT / name
            bdir.mkdir(parents=True, exist_ok=True)
            cpp_extension.load(
                name=name, sources=[str(src / f) for f in files],
                extra_cflags=CXX_FLAGS + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"],
                extra_cuda_cflags=NVCC_FLAGS + [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"],
                build_directory=str(bdir), verbose=verbose, is_python_module=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QIA_REFERENCE"),
                    help="reference checkout (holds third_party/sources/); or set QIA_REFERENCE")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    if not a.reference:
        ap.error("--reference (or QIA_REFERENCE) is required")
    print(build(Path(a.reference), a.force, a.verbose))
    sys.exit(0)
