// Shared helpers for the sm_100a kernels behind the qia_* C ABI.
//
// Every entry point validates its arguments on the host, launches on the
// caller's stream and returns a qia status code; it never aborts and never
// synchronises. The message of the last failure on the calling host thread is
// kept in a thread-local buffer (qia_last_error_string).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>
#include <math.h>

#include "../../include/qia_b200.h"

namespace qia {

// Records a formatted message as the thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);

// Checks the launch that was just queued; maps a CUDA error to QIA_ERR_CUDA.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Number of SMs of the current device (cached per device).
int sm_count();

// Device address of the library's device-side error word on the current
// device (bounded waits that give up write QIA_ERR_TIMEOUT there); nullptr
// if it cannot be resolved.
int* device_error_word();

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }
// Round an fp32 value through bf16 and back (the eager bf16 tensor boundary).
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// SiLU of a bf16 value as the reference's SwiGLU computes it
// (src/qwen_image_accel/kernels/bf16.py:12-24): div.rn(g, 1 + exp(-g)),
// rounded to bf16.
__device__ __forceinline__ float silu_ref(float g) { return round_bf16(__fdiv_rn(g, 1.0f + expf(-g))); }

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Unpack 8 bf16 values held in a uint4 into fp32.
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x);
  f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
  f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z);
  f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}

__device__ __forceinline__ void unpack4(const uint2& v, float* f) {
  f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x);
  f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
}

__device__ __forceinline__ uint2 pack4(const float* f) {
  uint2 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  return v;
}

// Two fp32 values -> two E4M3 codes (round to nearest even, saturate to +-448),
// low byte = first value.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ uint32_t cvt_e4m3x4(float a, float b, float c, float d) {
  return uint32_t(cvt_e4m3x2(a, b)) | (uint32_t(cvt_e4m3x2(c, d)) << 16);
}

// MXFP8 (OCP MX, E8M0 scale, 32-element blocks) exponent selection used by the
// reference quantizer (src/qwen_image_accel/kernels/mxfp8.py:46-50): the
// smallest power of two 2^(e-127) with amax / 2^(e-127) <= 448, read from the
// fp32 bits of amax; 0 when the block is all zeros; clamped to [0, 254].
__device__ __forceinline__ int mx_exponent(float amax) {
  const uint32_t bits = __float_as_uint(amax);
  int e = int((bits >> 23) & 0xffu) - 8 + (((bits & 0x7fffffu) > 6291456u) ? 1 : 0);
  e = e < 0 ? 0 : (e > 254 ? 254 : e);
  return amax == 0.0f ? 0 : e;
}

// 2^(127-e) as an exact fp32 bit pattern.
__device__ __forceinline__ float mx_inverse_scale(int e) {
  return __uint_as_float(uint32_t(254 - e) << 23);
}

// Byte offset of the E8M0 scale of (row, k-block) in the 128x4 blocked layout
// consumed by block-scaled tensor-core MMAs (reference kernels/mxfp8.py:53-56):
// 512-byte tiles of 128 rows x 4 k-blocks, ordered (row % 32, row / 32 % 4, kb % 4).
__host__ __device__ __forceinline__ int64_t mx_scale_offset(int64_t row, int64_t kb, int64_t kb_tiles) {
  return ((row >> 7) * kb_tiles + (kb >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (kb & 3);
}

// PyTorch's CUDA GELU (approximate="tanh") in fp32 opmath:
// 0.5*x*(1 + tanh(sqrt(2/pi) * (x + 0.044715*x^3))), with x^3 = (x*x)*x and the
// inner sum contracted to one fma.
__device__ __forceinline__ float gelu_tanh_f32(float x) {
  const float k_beta = float(M_SQRT2 * M_2_SQRTPI * 0.5);
  const float k_kappa = 0.044715f;
  const float x_cube = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(k_beta, __fmaf_rn(k_kappa, x_cube, x));
  return __fmul_rn(__fmul_rn(0.5f, x), 1.0f + tanhf(inner));
}

// The same GELU (tanh form) as x * sigmoid(2u), since 0.5 (1 + tanh u) =
// 1 / (1 + e^(-2u)): two MUFU operations (ex2, rcp; relative errors ~2^-22)
// instead of the accurate tanhf, and no cancellation for negative x. Within a
// few fp32 ulps of gelu_tanh_f32, so after bf16 rounding the two agree except
// at rounding boundaries. Used where the GELU sits in a GEMM epilogue.
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  // -2 * sqrt(2/pi) * log2(e)
  const float k_arg = float(-2.0 * M_SQRT2 * M_2_SQRTPI * 0.5 * 1.4426950408889634);
  const float k_kappa = 0.044715f;
  const float p = fmaf(k_kappa * (x * x), x, x);   // x + 0.044715 x^3
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(p * k_arg));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

// 256-bit global accesses (sm_100): one full 32-byte sector per instruction.
// The address must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* p, const uint4& a, const uint4& b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}
__device__ __forceinline__ void ld_global_v8(const void* p, uint4& a, uint4& b) {
  asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "l"(p));
}

// ---- packed fp32 pairs (sm_100 f32x2 FMA-pipe instructions): each lane of a
// pair is rounded exactly as the scalar instruction would round it.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// Both lanes rounded to bf16 (nearest even) and widened back to fp32.
__device__ __forceinline__ void round_bf16_x2(float& lo, float& hi) {
  uint32_t b;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b) : "f"(hi), "f"(lo));
  lo = __uint_as_float(b << 16);
  hi = __uint_as_float(b & 0xffff0000u);
}

// ---- packed bf16 pairs (low half = first element)
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Product of two bf16 pairs, rounded once to bf16: the exact product of two
// bf16 values fits an fp32 mantissa, so this equals bf16(fp32(a) * fp32(b))
// (for products down to 2^-135 in magnitude; smaller ones are zero or the
// smallest bf16 subnormal either way).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t abs_bf16x2(uint32_t a) { return a & 0x7fff7fffu; }

// Sum of two bf16 pairs rounded once to bf16: equals bf16(fp32(a) + fp32(b))
// (the fp32 sum is exact when the exponents differ by at most 16; beyond that
// the smaller operand is below half a bf16 ulp of the larger and both round to
// the larger).
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// gelu_tanh_fast on a pair: the same operations in the same order (so the
// same results), with the FMA-pipe steps issued as f32x2 instructions.
__device__ __forceinline__ void gelu_tanh_fast_x2(float& x0, float& x1) {
  const float k_arg = float(-2.0 * M_SQRT2 * M_2_SQRTPI * 0.5 * 1.4426950408889634);
  const float k_kappa = 0.044715f;
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t p = f2_fma(f2_mul(f2_pack(k_kappa, k_kappa), f2_mul(x, x)), x, x);
  float a0, a1, e0, e1, d0, d1, r0, r1;
  f2_unpack(f2_mul(p, f2_pack(k_arg, k_arg)), a0, a1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a1));
  f2_unpack(f2_add(f2_pack(1.0f, 1.0f), f2_pack(e0, e1)), d0, d1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
  f2_unpack(f2_mul(x, f2_pack(r0, r1)), x0, x1);
}

__device__ __forceinline__ float warp_max_xor(float v, int width_mask) {
  for (int o = width_mask; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace qia
