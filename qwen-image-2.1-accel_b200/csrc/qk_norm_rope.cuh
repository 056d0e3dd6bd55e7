// Per-head RMSNorm and complex RoPE on one 128-element head row held by 16
// lanes (8 contiguous elements per lane), shared by the attention-input kernels
// (attn_prep.cu) and the fused Sage quantizers (sage_attn.cu).
//
// Numerics (reference src/qwen_image_accel/kernels/attention.py:44-77,
// kernels/bf16.py:46-55, kernels/elementwise.py:37-60):
//  * RMSNorm over head_dim (= 128): normalised value rounded to bf16, then the
//    product with the bf16 weight rounded to bf16 (Diffusers RMSNorm order).
//  * RoPE on interleaved pairs (re, im) with the CUDA complex multiply's FMA
//    order: re' = fma(re, c, -(im * s)), im' = fma(im, c, re * s), then bf16.
#pragma once

#include "qia_common.cuh"

namespace qia {
namespace qkrows {

constexpr int kHeadDim = 128;
constexpr int kLanesPerRow = 16;

// 1 / RMS of the row held by the 16 lanes of this head row (each lane passes
// its 8 elements); only those 16 lanes take part: the two half-warps may be on
// different rows, loop trips or branches.
// Sum of squares in the order of PyTorch's CUDA mean(-1) over 128 fp32 values
// (the eager Diffusers RMSNorm): 32 vec4 partials ((a+b)+c)+d over contiguous
// groups, then a halving tree g[t] += g[t + w] for w = 16, 8, 4, 2, 1. Lane j
// of the 16-lane row group holds groups 2j (p0) and 2j+1 (p1): w = 16..2 pair
// lanes j and j^8, j^4, j^2, j^1; w = 1 is p0 + p1.
__device__ __forceinline__ float rms_inverse(const float (&f)[8], float eps) {
  const unsigned mask = 0xffffu << (threadIdx.x & 16);
  float p0 = ((f[0] * f[0] + f[1] * f[1]) + f[2] * f[2]) + f[3] * f[3];
  float p1 = ((f[4] * f[4] + f[5] * f[5]) + f[6] * f[6]) + f[7] * f[7];
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    p0 += __shfl_xor_sync(mask, p0, o);
    p1 += __shfl_xor_sync(mask, p1, o);
  }
  const float ss = p0 + p1;
  return rsqrtf(ss / float(kHeadDim) + eps);
}

__device__ __forceinline__ void rms_normalize(float (&f)[8], const float (&w)[8], float eps) {
  const float r = rms_inverse(f, eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(f[i], r)), w[i]));
}

// rms_normalize's scaling step, f[i] = bf16(bf16(f[i] * r) * w[i]), on f32x2
// pairs (each lane rounded as the scalar instructions round it).
__device__ __forceinline__ void rms_scale_x2(float (&f)[8], float r, const float (&w)[8]) {
  const uint64_t rr = f2_pack(r, r);
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float a, b;
    f2_unpack(f2_mul(f2_pack(f[i], f[i + 1]), rr), a, b);
    round_bf16_x2(a, b);
    f2_unpack(f2_mul(f2_pack(a, b), f2_pack(w[i], w[i + 1])), a, b);
    round_bf16_x2(a, b);
    f[i] = a;
    f[i + 1] = b;
  }
}

// freqs: [8 floats] = 4 (cos, sin) pairs for this thread's 4 complex pairs.
__device__ __forceinline__ void rope8(float (&f)[8], const float (&cs)[8]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float re = f[2 * p], im = f[2 * p + 1];
    const float c = cs[2 * p], s = cs[2 * p + 1];
    f[2 * p] = __fmaf_rn(re, c, -__fmul_rn(im, s));
    f[2 * p + 1] = __fmaf_rn(im, c, __fmul_rn(re, s));
  }
}

__device__ __forceinline__ void load_freqs(const float* __restrict__ freqs, int64_t token, int sub,
                                           float (&cs)[8]) {
  const float4* p = reinterpret_cast<const float4*>(freqs + token * kHeadDim + sub * 8);
  const float4 a = __ldg(p), b = __ldg(p + 1);
  cs[0] = a.x; cs[1] = a.y; cs[2] = a.z; cs[3] = a.w;
  cs[4] = b.x; cs[5] = b.y; cs[6] = b.z; cs[7] = b.w;
}

__device__ __forceinline__ void load_w(const __nv_bfloat16* __restrict__ w, int sub, float (&f)[8]) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(w + sub * 8)), f);
}

}  // namespace qkrows
}  // namespace qia
