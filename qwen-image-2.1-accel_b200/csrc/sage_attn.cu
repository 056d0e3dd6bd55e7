// Sage-style quantized attention on tcgen05: INT8 Q.K^T, FP8 P.V, online
// softmax in base 2, for the unmasked joint text+image attention.
//
// Semantics follow the reference's decode attention, sageattn_qk_int8_pv_fp8_cuda
// with qk_quant_gran="per_warp", pv_accum_dtype="fp32+fp32", smooth_k=True
// (reference src/qwen_image_accel/optimizations/sage_attention.py:19-25;
// SAGE:sageattention/core.py:725-828):
//  * K smoothing: k - mean_seq(k) (the mean rounded to bf16, core.py:773);
//  * Q INT8 per (32-token block, head), K INT8 per (64-token block, head):
//    scale = amax/127 (amax floored at 1e-7), codes = rint_sat(x * 127/amax)
//    (SAGE:csrc/fused/fused.cu:140-184);
//  * V FP8 E4M3 per (batch, head, channel): scale = amax/448
//    (SAGE:csrc/fused/fused.cu:316-427);
//  * the four divides (amax/127, 127/amax, amax/448, 448/amax) are
//    __fdividef: the reference extension is built with --use_fast_math
//    (SAGE:setup.py:53-61), under which its `/` is that intrinsic (the two
//    agree bit for bit on 4M quantizer-shaped divisions on a B200, and the
//    IEEE divide differs in ~30 % of them), so codes and scales match the
//    built reference bit for bit;
//  * S = int32 Q.K^T, s = S * (sm_scale*log2e) * (q_scale*k_scale); running
//    max m offset by log2(448) so P = 2^(s - m) lies in [0, 448]
//    (SAGE:csrc/qattn/attn_utils.cuh:353-440); P rounded to E4M3 for the
//    P.V product, the row sum taken over the unrounded P;
//  * the row max is found first: pass A computes Q.K^T for every K tile and
//    keeps only each row's max; pass B recomputes Q.K^T and forms
//    P = 2^(s - m) with the final m (offset by log2(448), so P <= 448 exactly
//    as in Sage), so no rescale of O is ever needed; P.V accumulates in a
//    full-fp32 TMEM accumulator. Sage's online form rounds P to E4M3 relative
//    to the running max instead; the two differ only for weights below
//    2^-9 of the row max;
//  * out = O / rowsum * v_scale, bf16 (SAGE:csrc/qattn/qk_int_sv_f8_cuda_sm89.cuh:566-600).
//
// Device layouts written by the quantization kernels here (head-major, rows
// padded to a multiple of 128 with zeros): q8/k8 int8 [B*H, S_pad, 128],
// v8 e4m3 [B*H, S_pad, 128], q_scale f32 [B*H, S_pad/32], k_scale f32
// [B*H, S_pad/64], v_scale f32 [B*H, 128], k_mean bf16 [B*H, 128]; scratch:
// v_recp f32 [B*H, 128], per-32-row-tile K sums and |V| maxima f32
// [B*H, S_pad/32, 128] each, normalised K bf16 [B*H, S_pad, 128] (joint
// entry points only).
#include <cudaTypedefs.h>

#include <climits>
#include <mutex>

#include "qk_norm_rope.cuh"
#include "sm100.cuh"

namespace qia {
namespace {

constexpr int kD = 128;
constexpr int kTile = 128;
constexpr int kKStages = 3;   // K tiles in flight (the row-max pass streams K only)
constexpr int kVStages = 2;
constexpr float kFp8Offset = 8.807f;  // log2(448): P = 2^(s - m) <= 448

// ------------------------------------------------------------------ quantizers
// Three launches fill the workspace.
//  1. sage_quant_q_stats_kernel, per (b, h, 32-row tile), 256 threads: Q codes
//     and scales (the tile is one Q block); per tile the column sums of K and
//     column maxima of |V|; for a source that normalises Q/K on load, also the
//     normalised K (bf16, in the workspace) for launch 3. Sixteen lanes per
//     row (eight channels each), sixteen rows per pass, two passes (row
//     p*16 + t/16 of the tile in pass p). Every thread first stages all the
//     16-byte pieces it will read (its Q/K/V row pieces and, with RoPE, its
//     32 bytes of each row's RoPE table) into shared memory with cp.async, so
//     the tile's loads are all in flight at once, then reads back only its own
//     pieces. K column sums: a thread adds its two rows in pass order to 0.0;
//     the two row groups of a warp (rows g and g+1 for even g) are added
//     (g + (g+1)); the eight warp sums are added in warp order to 0.0.
//  2. sage_quant_finalize_kernel, per (b, h): the tile partials reduced as
//     eight interleaved sub-sums (tiles j, j + 8, j + 16, ... in order), added
//     in sub order: k_mean = bf16(sum * (1/S)); v_scale = amax/448 and
//     v_recp = 448/amax (0 for an all-zero channel).
//  3. sage_quant_kv_kernel, per (b, h, 64-row tile) and z (0: K, 1: V): K
//     codes of k - k_mean in one 64-row block, or V E4M3 codes of
//     v * 448/amax, staged the same way (four passes).
// INT8 blocks: scale = amax/127 (amax floored at 1e-7), codes =
// rint_sat(x * 127/amax), both divides __fdividef; rows past S are zeros. The rows come from a source:
// strided [B, S, H, 128] bf16 tensors (PlainQKV), or the fused q|k|v
// projection outputs of the two streams of the joint [text, image] sequence
// (JointQKV), whose Q and K are normalised (per-head RMSNorm) and rotated
// (RoPE) on load with the roundings of the separate attention-input kernel.
constexpr int kQTile = 64;    // rows per K/V-quantization CTA (one K block)
constexpr int kQBlock = 32;   // rows per Q-statistics CTA (one Q block)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Q, K, V rows of [B, S, H, 128] bf16 tensors with element strides (b, s, h).
struct PlainQKV {
  static constexpr bool kNormRope = false;
  const __nv_bfloat16* x[3];
  int64_t sb[3], ss[3], sh[3];
  float eps;
  __device__ __forceinline__ const __nv_bfloat16* row(int c, int b, int h, int s) const {
    return x[c] + b * sb[c] + int64_t(s) * ss[c] + h * sh[c];
  }
  // The K rows the K-quantization launch reads (no normalised copy is kept).
  __device__ __forceinline__ const __nv_bfloat16* krow(int b, int h, int s) const { return row(1, b, h, s); }
  __device__ __forceinline__ __nv_bfloat16* knrow(int, int, int) const { return nullptr; }
  __device__ __forceinline__ const float* freqs(int) const { return nullptr; }
  __device__ __forceinline__ bool first(int) const { return true; }
  __device__ __forceinline__ uint4 weight(int, int) const { return make_uint4(0u, 0u, 0u, 0u); }
};

// The joint sequence: tokens [0, len0) from stream 0's projection output (rows
// b*len0 + s, leading dimension ld0; q at column 0, k at H*128, v at 2*H*128),
// tokens [len0, len0 + len1) from stream 1's; each stream's norm weights
// (wq*, wk*) and RoPE table (f*: [len, 64] (cos, sin) pairs). kn: the
// normalised K, [B*H, S_pad, 128] bf16, written by launch 1.
struct JointQKV {
  static constexpr bool kNormRope = true;
  const __nv_bfloat16* qkv0;
  const __nv_bfloat16* qkv1;
  int64_t ld0, ld1;
  const __nv_bfloat16* wq0;
  const __nv_bfloat16* wk0;
  const __nv_bfloat16* wq1;
  const __nv_bfloat16* wk1;
  const float* f0;
  const float* f1;
  __nv_bfloat16* kn;
  int len0, len1, H, S_pad;
  float eps;
  __device__ __forceinline__ const __nv_bfloat16* row(int c, int b, int h, int s) const {
    const bool first = s < len0;
    return (first ? qkv0 + (int64_t(b) * len0 + s) * ld0 : qkv1 + (int64_t(b) * len1 + (s - len0)) * ld1) +
           (int64_t(c) * H + h) * kD;
  }
  __device__ __forceinline__ __nv_bfloat16* knrow(int b, int h, int s) const {
    return kn + ((int64_t(b) * H + h) * S_pad + s) * kD;
  }
  __device__ __forceinline__ const __nv_bfloat16* krow(int b, int h, int s) const { return knrow(b, h, s); }
  __device__ __forceinline__ const float* freqs(int s) const {
    return s < len0 ? f0 + int64_t(s) * kD : f1 + int64_t(s - len0) * kD;
  }
  __device__ __forceinline__ bool first(int s) const { return s < len0; }
  // This lane's eight weights of component c (0 = q, 1 = k) of stream i.
  __device__ __forceinline__ uint4 weight(int c, int i) const {
    const __nv_bfloat16* w = c == 0 ? (i == 0 ? wq0 : wq1) : (i == 0 ? wk0 : wk1);
    return __ldg(reinterpret_cast<const uint4*>(w + (threadIdx.x & 15) * 8));
  }
};

// max(floor, |x_i|) over the eight bf16 values of a row piece.
__device__ __forceinline__ float piece_amax(const uint4& x, float floor) {
  const uint32_t m = max_bf16x2(max_bf16x2(abs_bf16x2(x.x), abs_bf16x2(x.y)),
                                max_bf16x2(abs_bf16x2(x.z), abs_bf16x2(x.w)));
  return fmaxf(floor, fmaxf(bf16_lo(m), bf16_hi(m)));
}

// RMSNorm (weight w, eps) + RoPE (cs = four (cos, sin) pairs) of a bf16 row
// piece, returned as bf16: the attention-input kernel's values
// (bf16(bf16(x * r) * w), then the complex product, then bf16), with the
// weight product as one bf16x2 multiply per pair.
__device__ __forceinline__ uint4 norm_rope_piece(const uint4& x, const uint4& w, const float (&cs)[8], float eps) {
  float f[8];
  unpack8(x, f);
  const float r = qkrows::rms_inverse(f, eps);
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t y = mul_bf16x2(cvt_bf16x2(__fmul_rn(f[2 * i], r), __fmul_rn(f[2 * i + 1], r)), wv[i]);
    const float re = bf16_lo(y), im = bf16_hi(y), c = cs[2 * i], s = cs[2 * i + 1];
    o[i] = cvt_bf16x2(__fmaf_rn(re, c, -__fmul_rn(im, s)), __fmaf_rn(im, c, __fmul_rn(re, s)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void load_cs(const uint4* sf0, const uint4* sf1, float (&cs)[8]) {
  const uint4 a = *sf0, b = *sf1;
  cs[0] = __uint_as_float(a.x); cs[1] = __uint_as_float(a.y); cs[2] = __uint_as_float(a.z);
  cs[3] = __uint_as_float(a.w); cs[4] = __uint_as_float(b.x); cs[5] = __uint_as_float(b.y);
  cs[6] = __uint_as_float(b.z); cs[7] = __uint_as_float(b.w);
}

// Maximum over the row's 16 lanes (xor shuffles stay inside the half-warp),
// and over the whole warp (both rows of a pass).
__device__ __forceinline__ float row_amax(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float pair_amax(float v) { return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16)); }

// INT8 codes rint(x * inv) of a bf16 row piece (minus mf when SUB_MEAN), four
// codes per 32-bit word. |x * inv| <= 127 * (1 + 2^-24)^2 < 127.5 because inv
// = 127/amax rounded and |x| <= amax, so no saturation is needed, and the
// rounding to an integer is done on the FMA pipe: adding 1.5 * 2^23 leaves
// round-to-nearest-even(x * inv) in the low mantissa bits (the same integer
// cvt.rni gives), whose low byte is the two's-complement code.
template <bool SUB_MEAN>
__device__ __forceinline__ uint2 int8_piece(const uint4& x, const float (&mf)[8], float inv) {
  constexpr float kMagic = 12582912.0f;
  float f[8];
  unpack8(x, f);
  uint32_t c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float v = SUB_MEAN ? __fsub_rn(f[e], mf[e]) : f[e];
    c[e] = __float_as_uint(__fadd_rn(__fmul_rn(v, inv), kMagic));
  }
  const uint32_t lo = __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
  const uint32_t hi = __byte_perm(__byte_perm(c[4], c[5], 0x0040), __byte_perm(c[6], c[7], 0x0040), 0x5410);
  return make_uint2(lo, hi);
}

// Dynamic shared memory of the staged kernels (16-byte slots, one per thread).
template <class Src>
constexpr int q_stats_smem() {
  return (3 + (Src::kNormRope ? 2 : 0)) * 2 * 256 * 16;
}
constexpr int kKvSmem = 4 * 256 * 16;

// Grid (B*H, max(Sq_pad/32, ceil(Skv/32))), 256 threads: one 32-row tile,
// two passes.
template <class Src>
__global__ void __launch_bounds__(256, 4) sage_quant_q_stats_kernel(Src src, int Sq, int Sq_pad, int Skv, int H,
                                                                    int kv_tiles, int part_stride,
                                                                    int8_t* __restrict__ q8,
                                                                    float* __restrict__ q_scale,
                                                                    float* __restrict__ k_part,
                                                                    float* __restrict__ v_part) {
  extern __shared__ __align__(16) uint4 q_stage[];
  __shared__ __align__(16) float s_k[8][kD];
  __shared__ __align__(16) float s_v[8][kD];
  __shared__ __align__(16) float s_wmax[8];
  const int bh = blockIdx.x, b = bh / H, h = bh % H, tile = blockIdx.y, t = threadIdx.x;
  const int cg = t & 15, rs = t >> 4, warp = t >> 5;
  const bool do_q = tile * kQBlock < Sq_pad, do_kv = tile < kv_tiles;
  // slots: x[c][p][t] (c = q, k, v), then the rows' RoPE pieces f[half][p][t]
  // (Q and K of a row share them; a source with RoPE has Sq == Skv)
  auto sx = [&](int c, int p) { return q_stage + (c * 2 + p) * 256 + t; };
  auto sf = [&](int half, int p) { return q_stage + 3 * 2 * 256 + (half * 2 + p) * 256 + t; };
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int row = tile * kQBlock + p * 16 + rs;
    const bool vq = row < Sq, vkv = row < Skv;
    cp_async16(sx(0, p), (vq ? src.row(0, b, h, row) : src.row(0, 0, 0, 0)) + cg * 8, vq);
    cp_async16(sx(1, p), (vkv ? src.row(1, b, h, row) : src.row(1, 0, 0, 0)) + cg * 8, vkv);
    cp_async16(sx(2, p), (vkv ? src.row(2, b, h, row) : src.row(2, 0, 0, 0)) + cg * 8, vkv);
    if (Src::kNormRope) {
      const float* f = (vq ? src.freqs(row) : src.freqs(0)) + cg * 8;
      cp_async16(sf(0, p), f, vq);
      cp_async16(sf(1, p), f + 4, vq);
    }
  }
  cp_async_wait_all();
  uint4 qx[2];
  float ks[8];
  uint32_t vm2[4] = {0u, 0u, 0u, 0u};
  float amax = 1e-7f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ks[e] = 0.0f;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int row = tile * kQBlock + p * 16 + rs;
    float cs[8];
    const int stream = src.first(row) ? 0 : 1;
    if (Src::kNormRope) load_cs(sf(0, p), sf(1, p), cs);
    qx[p] = make_uint4(0u, 0u, 0u, 0u);
    if (row < Sq) {
      qx[p] = *sx(0, p);
      if (Src::kNormRope) qx[p] = norm_rope_piece(qx[p], src.weight(0, stream), cs, src.eps);
      amax = piece_amax(qx[p], amax);
    }
    if (row < Skv) {
      uint4 y = *sx(1, p);
      if (Src::kNormRope) {
        y = norm_rope_piece(y, src.weight(1, stream), cs, src.eps);
        *reinterpret_cast<uint4*>(src.knrow(b, h, row) + cg * 8) = y;
      }
      float f[8];
      unpack8(y, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ks[e] += f[e];
      const uint4 v = *sx(2, p);
      vm2[0] = max_bf16x2(vm2[0], abs_bf16x2(v.x));
      vm2[1] = max_bf16x2(vm2[1], abs_bf16x2(v.y));
      vm2[2] = max_bf16x2(vm2[2], abs_bf16x2(v.z));
      vm2[3] = max_bf16x2(vm2[3], abs_bf16x2(v.w));
    }
  }
  // the tile is one 32-row Q block: per warp (both half-warps), then across warps
  amax = pair_amax(row_amax(amax));
  if ((t & 31) == 0) s_wmax[warp] = amax;
  // K sums / |V| maxima: the two row groups of a warp combined (one add), then
  // the eight warps in order through shared memory
  float vm[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    vm[2 * i] = bf16_lo(vm2[i]);
    vm[2 * i + 1] = bf16_hi(vm2[i]);
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], 16);
    vm[e] = fmaxf(vm[e], __shfl_xor_sync(0xffffffffu, vm[e], 16));
  }
  if (rs % 2 == 0) {
    float4* sk = reinterpret_cast<float4*>(&s_k[warp][cg * 8]);
    float4* sv = reinterpret_cast<float4*>(&s_v[warp][cg * 8]);
    sk[0] = make_float4(ks[0], ks[1], ks[2], ks[3]);
    sk[1] = make_float4(ks[4], ks[5], ks[6], ks[7]);
    sv[0] = make_float4(vm[0], vm[1], vm[2], vm[3]);
    sv[1] = make_float4(vm[4], vm[5], vm[6], vm[7]);
  }
  __syncthreads();
  if (t < kD && do_kv) {
    float sum = 0.0f, vmax = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      sum += s_k[w][t];
      vmax = fmaxf(vmax, s_v[w][t]);
    }
    const int64_t o = (int64_t(bh) * part_stride + tile) * kD + t;
    k_part[o] = sum;
    v_part[o] = vmax;
  }
  if (!do_q) return;
  const float4 a = *reinterpret_cast<const float4*>(&s_wmax[0]);
  const float4 c = *reinterpret_cast<const float4*>(&s_wmax[4]);
  const float bm = fmaxf(fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)), fmaxf(fmaxf(c.x, c.y), fmaxf(c.z, c.w)));
  if (t == 0) q_scale[int64_t(bh) * (Sq_pad / 32) + tile] = __fdividef(bm, 127.0f);
  const float inv = __fdividef(127.0f, bm);
  const float none[8] = {};
  int8_t* dst = q8 + (int64_t(bh) * Sq_pad + tile * kQBlock) * kD + cg * 8;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int r = p * 16 + rs;
    const uint2 code = tile * kQBlock + r < Sq ? int8_piece<false>(qx[p], none, inv) : make_uint2(0u, 0u);
    *reinterpret_cast<uint2*>(dst + int64_t(r) * kD) = code;
  }
}

// Grid (B*H, 4), 256 threads: 32 channels per CTA, eight sub-sums per
// channel. Thread (sub, channel) adds the partials of tiles sub, sub + 8,
// sub + 16, ... in order to 0.0 (all its loads in flight at once, 16 at a
// time); the eight sub-sums are then added in sub order to 0.0. |V| maxima
// the same way.
__global__ void __launch_bounds__(256) sage_quant_finalize_kernel(const float* __restrict__ k_part,
                                                                  const float* __restrict__ v_part, int tiles,
                                                                  int part_stride, int S,
                                                                  __nv_bfloat16* __restrict__ k_mean,
                                                                  float* __restrict__ v_scale,
                                                                  float* __restrict__ v_recp) {
  __shared__ float s_sum[8][32], s_max[8][32];
  const int bh = blockIdx.x, t = threadIdx.x, ch = t & 31, sub = t >> 5, d = blockIdx.y * 32 + ch;
  const int64_t base = int64_t(bh) * part_stride * kD + d;
  float sum = 0.0f, amax = 0.0f;
  for (int i0 = sub; i0 < tiles; i0 += 8 * 16) {
    float kv[16], vv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int i = i0 + 8 * j;
      kv[j] = i < tiles ? __ldg(k_part + base + int64_t(i) * kD) : 0.0f;
      vv[j] = i < tiles ? __ldg(v_part + base + int64_t(i) * kD) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (i0 + 8 * j < tiles) {
        sum += kv[j];
        amax = fmaxf(amax, vv[j]);
      }
    }
  }
  s_sum[sub][ch] = sum;
  s_max[sub][ch] = amax;
  __syncthreads();
  if (t < 32) {
    float total = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) total += s_sum[j][ch];
    k_mean[int64_t(bh) * kD + d] = __float2bfloat16_rn(total * (1.0f / float(S)));
  } else if (t < 64) {
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, s_max[j][ch]);
    v_scale[int64_t(bh) * kD + d] = __fdividef(m, 448.0f);
    v_recp[int64_t(bh) * kD + d] = m > 0.0f ? __fdividef(448.0f, m) : 0.0f;
  }
}

// Grid (B*H, S_pad/64, 2), 256 threads. z = 0: K codes of k - k_mean (one
// 64-row block per tile); z = 1: V codes of v * 448/amax.
template <class Src>
__global__ void __launch_bounds__(256, 4) sage_quant_kv_kernel(Src src, int S, int S_pad, int H,
                                                               const __nv_bfloat16* __restrict__ k_mean,
                                                               const float* __restrict__ v_recp,
                                                               int8_t* __restrict__ k8, float* __restrict__ k_scale,
                                                               uint8_t* __restrict__ v8) {
  extern __shared__ __align__(16) uint4 kv_stage[];
  __shared__ __align__(16) float s_wmax[8];
  const int bh = blockIdx.x, b = bh / H, h = bh % H, tile = blockIdx.y, t = threadIdx.x;
  const int cg = t & 15, rs = t >> 4, warp = t >> 5;
  const bool is_k = blockIdx.z == 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int row = tile * kQTile + p * 16 + rs;
    const bool valid = row < S;
    const __nv_bfloat16* g = is_k ? (valid ? src.krow(b, h, row) : src.krow(0, 0, 0))
                                  : (valid ? src.row(2, b, h, row) : src.row(2, 0, 0, 0));
    cp_async16(kv_stage + p * 256 + t, g + cg * 8, valid);
  }
  float cc[8];
  if (is_k) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(k_mean + int64_t(bh) * kD + cg * 8)), cc);
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(v_recp + int64_t(bh) * kD + cg * 8));
    const float4 c = __ldg(reinterpret_cast<const float4*>(v_recp + int64_t(bh) * kD + cg * 8 + 4));
    cc[0] = a.x; cc[1] = a.y; cc[2] = a.z; cc[3] = a.w; cc[4] = c.x; cc[5] = c.y; cc[6] = c.z; cc[7] = c.w;
  }
  cp_async_wait_all();
  if (is_k) {
    uint4 kx[4];
    float rmax = 1e-7f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      kx[p] = kv_stage[p * 256 + t];
      if (tile * kQTile + p * 16 + rs < S) {
        float f[8];
        unpack8(kx[p], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) rmax = fmaxf(rmax, fabsf(f[e] - cc[e]));
      }
    }
    rmax = pair_amax(row_amax(rmax));
    if ((t & 31) == 0) s_wmax[warp] = rmax;
    __syncthreads();
    const float4 a = *reinterpret_cast<const float4*>(&s_wmax[0]);
    const float4 c = *reinterpret_cast<const float4*>(&s_wmax[4]);
    const float bm = fmaxf(fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)), fmaxf(fmaxf(c.x, c.y), fmaxf(c.z, c.w)));
    if (t == 0) k_scale[int64_t(bh) * (S_pad / 64) + tile] = __fdividef(bm, 127.0f);
    const float inv = __fdividef(127.0f, bm);
    int8_t* dst = k8 + (int64_t(bh) * S_pad + tile * kQTile) * kD + cg * 8;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int r = p * 16 + rs;
      const uint2 code = tile * kQTile + r < S ? int8_piece<true>(kx[p], cc, inv) : make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(dst + int64_t(r) * kD) = code;
    }
    return;
  }
  uint8_t* dst = v8 + (int64_t(bh) * S_pad + tile * kQTile) * kD + cg * 8;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    float f[8];
    unpack8(kv_stage[p * 256 + t], f);      // zero-filled past S
    const uint32_t lo = cvt_e4m3x4(f[0] * cc[0], f[1] * cc[1], f[2] * cc[2], f[3] * cc[3]);
    const uint32_t hi = cvt_e4m3x4(f[4] * cc[4], f[5] * cc[5], f[6] * cc[6], f[7] * cc[7]);
    *reinterpret_cast<uint2*>(dst + int64_t(p * 16 + rs) * kD) = make_uint2(lo, hi);
  }
}

// ------------------------------------------------------------------ attention
// Instruction descriptors (tcgen05 kind::i8 and kind::f8f6f4, M = N = 128).
constexpr uint32_t kIdescQK = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTile >> 3) << 17) |
                              (uint32_t(128 >> 4) << 24);  // s32 accum, s8 x s8, K-major both
constexpr uint32_t kIdescPV = (1u << 4) | (0u << 7) | (0u << 10) | (1u << 16) | (uint32_t(kD >> 3) << 17) |
                              (uint32_t(128 >> 4) << 24);  // f32 accum, e4m3 x e4m3, B (V) MN-major

__device__ __forceinline__ void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// MN-major, 128-byte swizzle descriptor (V as the B operand of P.V): 128 B of
// N per row, 8-row (K) groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// int32 (|x| < 2^22) -> fp32 exactly, on the FMA/ALU pipes.
__device__ __forceinline__ float i2f_small(uint32_t x) {
  return __int_as_float(int(x) + 0x4B400000) - 12582912.0f;
}

struct AttnParams {
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  __nv_bfloat16* out;       // NHD [B, split, H, 128]: query tokens [0, split)
  int64_t out_stride_b, out_stride_s, out_stride_h;
  __nv_bfloat16* out2;      // NHD [B, Sq - split, H, 128]: query tokens [split, Sq)
  int64_t out2_stride_b, out2_stride_s, out2_stride_h;
  int split;
  int B, H, Sq, Skv, Sq_pad, Skv_pad;
  float sm_scale_log2;      // sm_scale * log2(e)
  // MXFP8 output (instead of bf16): the two streams as E4M3 rows [tokens, H*128]
  // with E8M0 scales in the 128x4 blocked layout -- the next GEMM's operand
  uint8_t* qa_values;       // null: bf16 output through out / out2
  uint8_t* qa_scales;
  uint8_t* qb_values;
  uint8_t* qb_scales;
  // Optional per-query key limit (block-causal prefill): query token t of
  // batch b attends to keys [0, kv_limit[b * kv_limit_stride_b + t]) only,
  // clamped to [0, Skv]. Null: every query sees all Skv keys.
  const int* kv_limit;
  int64_t kv_limit_stride_b;
  // Ulysses output exchange (null img_peers: the outputs above). Batch 1: the
  // image row j of the joint sequence (query token split + j) goes straight to
  // the rank that owns the token -- row j % peer_rows of img_peers[j /
  // peer_rows] -- and every text row to each rank's txt_peers buffer, both
  // [rows, peer_ld] bf16 at columns (peer_head0 + h) * 128. After its stores
  // every CTA adds 1 to counter peer_slot of each rank (signal_peers), after a
  // system-scope fence.
  __nv_bfloat16* const* img_peers;
  __nv_bfloat16* const* txt_peers;
  unsigned long long* const* signal_peers;
  int peer_count, peer_rows, peer_head0, peer_slot;
  int64_t peer_ld;
};

// Two CTAs share an SM (98 KB of shared memory and 256 TMEM columns each), so
// one CTA's MMAs run while the other's softmax warps work.
//
// TMEM columns of a CTA:
//   row-max pass: S buffers [0,128) and [128,256), alternating per K tile;
//   P pass:       S halves of 64 keys at [0,64) and [64,128), alternating; P of
//                 a half (E4M3, 4 per column) overwrites the first 16 columns
//                 of its own S half and is the TMEM A operand of P.V; the O
//                 accumulator is [128,256).
// MMAs issued by one thread execute in issue order, so the Q.K^T that reuses
// an S half is issued right after the P.V that reads the P stored there.
constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + 16384;
constexpr int kSmemV = kSmemK + kKStages * 16384;
constexpr int kSmemBar = kSmemV + kVStages * 16384;
constexpr int kAttnSmem = kSmemBar + 1024 + 1024;
constexpr uint32_t kAttnTmemCols = 256;
constexpr uint32_t kTmemO = 128;
constexpr int kHalf = 64;   // keys per S half in the P pass (= one K scale block)
constexpr uint32_t kIdescQK64 = (kIdescQK & ~(0x3Fu << 17)) | (uint32_t(kHalf >> 3) << 17);

__device__ __forceinline__ void tc_mma_f8_tmem_a(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                                 uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tc_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// P of one 64-key half for one query row: P = 2^(S * sc - m) (S the int32
// scores of the half, m the row max offset by log2(448), so P <= 448) as E4M3
// codes four per word into w, the fp32 P added to the row sum (lane pairs
// ds01 / ds23 on the full path, ds[] on a ragged last half of `valid` keys).
__device__ __forceinline__ void p_half(const uint32_t (&sv)[64], int valid, float sc, float m, uint64_t& ds01,
                                       uint64_t& ds23, float (&ds)[4], uint32_t (&w)[16]) {
  if (valid >= kHalf) {
    // s*sc - m = X*sc - (2^23+2^22)*sc - m with X = float(2^23+2^22+s)
    // exactly (|s| < 2^22): one FMA per score after an integer add
    const float bias = fmaf(12582912.0f, sc, m);
    const uint64_t sc2 = f2_pack(sc, sc), nb2 = f2_pack(-bias, -bias);
#pragma unroll
    for (int t4 = 0; t4 < 64; t4 += 4) {
      float a[4], pv[4];
      f2_unpack(f2_fma(f2_pack(__int_as_float(int(sv[t4]) + 0x4B400000), __int_as_float(int(sv[t4 + 1]) + 0x4B400000)),
                       sc2, nb2), a[0], a[1]);
      f2_unpack(f2_fma(f2_pack(__int_as_float(int(sv[t4 + 2]) + 0x4B400000), __int_as_float(int(sv[t4 + 3]) + 0x4B400000)),
                       sc2, nb2), a[2], a[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) pv[e] = ex2_approx(a[e]);
      ds01 = f2_add(ds01, f2_pack(pv[0], pv[1]));
      ds23 = f2_add(ds23, f2_pack(pv[2], pv[3]));
      w[t4 / 4] = cvt_e4m3x4(pv[0], pv[1], pv[2], pv[3]);
    }
  } else {
#pragma unroll
    for (int t4 = 0; t4 < 64; t4 += 4) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[e] = t4 + e < valid ? ex2_approx(fmaf(i2f_small(sv[t4 + e]), sc, -m)) : 0.0f;
        ds[e] += pv[e];
      }
      w[t4 / 4] = cvt_e4m3x4(pv[0], pv[1], pv[2], pv[3]);
    }
  }
}

// The epilogue of one query row (one thread, its TMEM lane): O (128 fp32
// columns from o_col) / rowsum * v_scale -> the bf16 output row (stream a or
// b of the joint sequence) or, with MXFP8 outputs, its E4M3 codes and E8M0
// scales. A row that saw no key (rowsum 0) writes zeros.
__device__ __forceinline__ void attn_store_row(const AttnParams& p, uint32_t tmem, uint32_t t_lane, uint32_t o_col,
                                               int bh, int q_tok, float dsum) {
  // a row that may see no key at all (a key limit of 0) writes zeros
  const float rinv = dsum > 0.0f ? 1.0f / dsum : 0.0f;
  const float* vs = p.v_scale + int64_t(bh) * kD;
  const int b = bh / p.H, h = bh % p.H;
  if (p.qa_values) {
    // bf16(O * rinv * v_scale) quantized to MXFP8 in place of the bf16 store:
    // this thread's 128 channels of head h are four 32-wide MX blocks of row
    // `row` of its stream, K index 128 h .. 128 h + 127 of the next GEMM
    const bool in_a = q_tok < p.split;
    const int64_t len = in_a ? p.split : p.Sq - p.split;
    const int64_t row = int64_t(b) * len + (in_a ? q_tok : q_tok - p.split);
    uint8_t* qv = (in_a ? p.qa_values : p.qb_values) + row * int64_t(p.H * kD) + h * kD;
    uint8_t* qsc = in_a ? p.qa_scales : p.qb_scales;
    uint32_t e4 = 0;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t ov[32];
      tc_ld_32x32b_x32(tmem + t_lane + o_col + uint32_t(c * 32), ov);
      tc_wait_ld();
      float f[32];
      float amax = 0.0f;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        f[e] = round_bf16(__uint_as_float(ov[e]) * rinv * __ldg(vs + c * 32 + e));
        amax = fmaxf(amax, fabsf(f[e]));
      }
      const int ex = mx_exponent(amax);
      const float inv = mx_inverse_scale(ex);
      uint32_t w[8];
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4)
        w[q4] = cvt_e4m3x4(f[4 * q4] * inv, f[4 * q4 + 1] * inv, f[4 * q4 + 2] * inv, f[4 * q4 + 3] * inv);
      if (q_tok < p.Sq)
        st_global_v8(qv + c * 32, make_uint4(w[0], w[1], w[2], w[3]), make_uint4(w[4], w[5], w[6], w[7]));
      e4 |= uint32_t(ex) << (8 * c);
    }
    // the four scale bytes (K blocks 4h .. 4h+3) are adjacent in the blocked layout
    if (q_tok < p.Sq) *reinterpret_cast<uint32_t*>(qsc + mx_scale_offset(row, 4 * h, p.H)) = e4;
  } else if (p.img_peers) {
    // Ulysses: an image row to the rank that owns its token, a text row to
    // every rank (NVLink stores into the peers' buffers)
    const int64_t col = int64_t(p.peer_head0 + h) * kD;
    const bool txt = q_tok < p.split;
    const int j = q_tok - p.split;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t ov[32];
      tc_ld_32x32b_x32(tmem + t_lane + o_col + uint32_t(c * 32), ov);
      tc_wait_ld();
      if (q_tok < p.Sq) {
        uint4 pk[4];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            f[e] = __uint_as_float(ov[c8 * 8 + e]) * rinv * __ldg(vs + c * 32 + c8 * 8 + e);
          pk[c8] = pack8(f);
        }
        if (txt) {
          for (int r = 0; r < p.peer_count; ++r) {
            uint4* dst = reinterpret_cast<uint4*>(p.txt_peers[r] + int64_t(q_tok) * p.peer_ld + col) + c * 4;
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) dst[c8] = pk[c8];
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(p.img_peers[j / p.peer_rows] + int64_t(j % p.peer_rows) * p.peer_ld +
                                                col) + c * 4;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) dst[c8] = pk[c8];
        }
      }
    }
  } else {
  // the joint [text, image] sequence can be written back as two streams
  uint4* dst = q_tok < p.split
                   ? reinterpret_cast<uint4*>(p.out + b * p.out_stride_b + int64_t(q_tok) * p.out_stride_s +
                                              h * p.out_stride_h)
                   : reinterpret_cast<uint4*>(p.out2 + b * p.out2_stride_b +
                                              int64_t(q_tok - p.split) * p.out2_stride_s + h * p.out2_stride_h);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t ov[32];
    tc_ld_32x32b_x32(tmem + t_lane + o_col + uint32_t(c * 32), ov);
    tc_wait_ld();
    if (q_tok < p.Sq) {
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          f[e] = __uint_as_float(ov[c8 * 8 + e]) * rinv * __ldg(vs + c * 32 + c8 * 8 + e);
        dst[c * 4 + c8] = pack8(f);
      }
    }
  }
  }
}

__global__ void __launch_bounds__(192, 2)
sage_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, AttnParams p, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* sa_full = v_empty + kVStages;  // [2] row-max pass: S buffer b written (one phase per use)
  uint64_t* sa_free = sa_full + 2;          // [2] row-max pass: S buffer b read by the softmax warps
  uint64_t* sb_full = sa_free + 2;          // [2] P pass: S half h written
  uint64_t* pb_full = sb_full + 2;          // [2] P pass: P of half h stored (S half h consumed)
  uint64_t* o_full = pb_full + 2;           // all P.V done
  uint64_t* drain = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* kv_extent = reinterpret_cast<int*>(tmem_slot + 1);   // largest key limit of this query tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // with key limits the grid is (B*H, query tiles) and the last query tiles,
  // which see the most keys, are issued first (longest first shortens the tail)
  const int q_tile = p.kv_limit ? int(gridDim.y - 1 - blockIdx.y) : int(blockIdx.x);
  const int bh = p.kv_limit ? int(blockIdx.x) : int(blockIdx.y);
  int nkv = p.Skv_pad / kTile;
  const int q_row0 = bh * p.Sq_pad + q_tile * kTile;
  const int kv_row0 = bh * p.Skv_pad;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&sa_full[b]), 1);
      mbar_init(smem_u32(&sa_free[b]), 4);
      mbar_init(smem_u32(&sb_full[b]), 1);
      mbar_init(smem_u32(&pb_full[b]), 4);
    }
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(drain), 1);
    *kv_extent = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), kAttnTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // this thread's key limit when it is a softmax thread (one query row each)
  int kv_lim = p.Skv;
  if (p.kv_limit) {
    // the tile visits only the key tiles its rows may see
    if (warp >= 2) {
      const int q_tok = q_tile * kTile + (warp & 3) * 32 + lane;
      kv_lim = q_tok < p.Sq ? min(max(__ldg(p.kv_limit + (bh / p.H) * p.kv_limit_stride_b + q_tok), 0), p.Skv) : 0;
      const int wmax = __reduce_max_sync(0xffffffffu, kv_lim);
      if (lane == 0) atomicMax(kv_extent, wmax);
    }
    __syncthreads();
    nkv = max(1, (*kv_extent + kTile - 1) / kTile);
  }
  const int nh = 2 * nkv;                   // 64-key halves in the P pass

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      int issued = 0, issued_v = 0;
      mbar_arrive_expect_tx(smem_u32(q_full), 16384);
      tma_load_2d(smem_u32(smem + kSmemQ), &tm_q, smem_u32(q_full), 0, q_row0);
      // steps [0, nkv): K tiles for the row-max pass; [nkv, 2 nkv): K and V tiles
      for (int t = 0; t < 2 * nkv && ok; ++t) {
        const int j = t < nkv ? t : t - nkv;
        const int st = t % kKStages;
        const uint32_t ph = (t / kKStages) & 1;
        if (!mbar_wait(smem_u32(&k_empty[st]), ph ^ 1, err)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_u32(&k_full[st]), 16384);
        tma_load_2d(smem_u32(smem + kSmemK + st * 16384), &tm_k, smem_u32(&k_full[st]), 0, kv_row0 + j * kTile);
        if (t >= nkv) {
          const int vs = j % kVStages;
          const uint32_t vph = (j / kVStages) & 1;
          if (!mbar_wait(smem_u32(&v_empty[vs]), vph ^ 1, err)) { ok = false; break; }
          mbar_arrive_expect_tx(smem_u32(&v_full[vs]), 16384);
          tma_load_2d(smem_u32(smem + kSmemV + vs * 16384), &tm_v, smem_u32(&v_full[vs]), 0, kv_row0 + j * kTile);
          issued_v = j + 1;
        }
        issued = t + 1;
      }
      if (!ok) {
        // let queued copies land before the shared memory is released
        mbar_wait(smem_u32(q_full), 0, nullptr, 100000000ull);
        for (int t = (issued > kKStages ? issued - kKStages : 0); t < issued; ++t)
          mbar_wait(smem_u32(&k_full[t % kKStages]), (t / kKStages) & 1, nullptr, 100000000ull);
        for (int j = (issued_v > kVStages ? issued_v - kVStages : 0); j < issued_v; ++j)
          mbar_wait(smem_u32(&v_full[j % kVStages]), (j / kVStages) & 1, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(smem_u32(q_full), 0, err);
      tc_fence_after();
      const uint64_t qdesc = smem_desc_k_sw128(smem_u32(smem + kSmemQ));
      // ---- row-max pass: Q.K^T of K tile j into S buffer j&1
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j % kKStages, b = j & 1, u = j >> 1;
        if (!mbar_wait(smem_u32(&k_full[st]), (j / kKStages) & 1, err)) { ok = false; break; }
        // buffer b is free once the softmax read its previous use (phase u-1)
        if (!mbar_wait(smem_u32(&sa_free[b]), (u & 1) ^ 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint64_t kdesc = smem_desc_k_sw128(smem_u32(smem + kSmemK + st * 16384));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_i8(tmem + uint32_t(b * 128), qdesc + uint64_t(2 * kk), kdesc + uint64_t(2 * kk), kIdescQK, kk > 0);
        tc_commit(smem_u32(&k_empty[st]));
        tc_commit(smem_u32(&sa_full[b]));
      }
      // ---- P pass. The S halves overwrite S buffer 0 of the row-max pass:
      // wait for the softmax's read of its last use there (use ua-1). Buffer 1
      // (O) is free once P of half 0 arrives, which follows the whole pass.
      const int ua = (nkv + 1) / 2;
      if (ok && !mbar_wait(smem_u32(&sa_free[0]), (ua & 1) ^ 1, err)) ok = false;
      tc_fence_after();
      // Q.K^T of half i (keys [64 i, 64 i + 64)) into S half i&1
      auto qk_half = [&](int i) -> bool {
        const int h = i & 1, t = nkv + (i >> 1), st = t % kKStages;
        if (h == 0) {
          if (!mbar_wait(smem_u32(&k_full[st]), (t / kKStages) & 1, err)) return false;
          tc_fence_after();
        }
        // rows [64 h, 64 h + 64) of the K tile start 8 KB in (8-row groups of 1 KB)
        const uint64_t kdesc = smem_desc_k_sw128(smem_u32(smem + kSmemK + st * 16384 + h * 8192));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_i8(tmem + uint32_t(h * kHalf), qdesc + uint64_t(2 * kk), kdesc + uint64_t(2 * kk), kIdescQK64,
                    kk > 0);
        tc_commit(smem_u32(&sb_full[h]));
        if (h == 1) tc_commit(smem_u32(&k_empty[st]));
        return true;
      };
      // O += P(half i) . V(keys of half i); A (P) from TMEM
      auto pv_half = [&](int i) -> bool {
        const int h = i & 1, jv = i >> 1, vs = jv % kVStages;
        if (!mbar_wait(smem_u32(&pb_full[h]), (i >> 1) & 1, err)) return false;
        if (h == 0 && !mbar_wait(smem_u32(&v_full[vs]), (jv / kVStages) & 1, err)) return false;
        tc_fence_after();
        const uint64_t vdesc = smem_desc_mn_sw128(smem_u32(smem + kSmemV + vs * 16384));
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          tc_mma_f8_tmem_a(tmem + kTmemO, tmem + uint32_t(h * kHalf + 8 * kk), vdesc + uint64_t(256 * (2 * h + kk)),
                           kIdescPV, (i | kk) != 0);
        if (h == 1) tc_commit(smem_u32(&v_empty[vs]));
        return true;
      };
      if (ok) ok = qk_half(0);
      if (ok) ok = qk_half(1);
      for (int i = 0; i < nh && ok; ++i) {
        ok = pv_half(i);
        if (ok && i + 2 < nh) ok = qk_half(i + 2);
      }
      if (ok) tc_commit(smem_u32(o_full));
      tc_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, ok ? err : nullptr, 100000000ull);
    }
  } else {
    // ---------------------------------------------------------- softmax
    // One thread per query row (TMEM lane).
    const int sub = warp & 3;
    const int r = sub * 32 + lane;            // row within the query tile
    const int q_tok = q_tile * kTile + r;     // token index
    const uint32_t t_lane = uint32_t(sub * 32) << 16;
    const float qs = p.q_scale[int64_t(bh) * (p.Sq_pad / 32) + q_tok / 32];
    const int kb_per_head = p.Skv_pad / 64;
    bool ok = true;
    // ---- row-max pass: the row max of s = S * (sm_scale*log2e) * (q_scale*k_scale)
    // (the two K-block scales of a tile are fetched one tile ahead)
    const float* ks_head = p.k_scale + int64_t(bh) * kb_per_head;
    const float qsl = p.sm_scale_log2 * qs;
    float2 ks_next = make_float2(__ldg(ks_head), __ldg(ks_head + 1));
    float m = -5000000.0f;
    for (int j = 0; j < nkv; ++j) {
      const float sc0 = qsl * ks_next.x, sc1 = qsl * ks_next.y;
      const int jn = j + 1 < nkv ? j + 1 : 0;
      ks_next = make_float2(__ldg(ks_head + 2 * jn), __ldg(ks_head + 2 * jn + 1));
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&sa_full[j & 1]), (j >> 1) & 1, err))) { ok = false; break; }
      tc_fence_after();
      const int valid = kv_lim - j * kTile;
      uint32_t sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tc_ld_32x32b_x32(tmem + t_lane + uint32_t((j & 1) * 128 + c * 32),
                         *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sa_free[j & 1]));
      int mx[2];
      if (valid >= kTile) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          // four independent chains, then a 4-way merge
          const uint32_t* x = sv + h2 * 64;
          int c0 = int(x[0]), c1 = int(x[1]), c2 = int(x[2]), c3 = int(x[3]);
#pragma unroll
          for (int t = 4; t < 60; t += 8) {   // x[4..59]
            c0 = __vimax3_s32(c0, int(x[t]), int(x[t + 1]));
            c1 = __vimax3_s32(c1, int(x[t + 2]), int(x[t + 3]));
            c2 = __vimax3_s32(c2, int(x[t + 4]), int(x[t + 5]));
            c3 = __vimax3_s32(c3, int(x[t + 6]), int(x[t + 7]));
          }
          c0 = __vimax3_s32(c0, int(x[60]), int(x[61]));
          c1 = __vimax3_s32(c1, int(x[62]), int(x[63]));
          mx[h2] = max(__vimax3_s32(c0, c1, c2), c3);
        }
      } else {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          int mh = INT_MIN;
#pragma unroll
          for (int t = 0; t < 64; ++t)
            if (h2 * 64 + t < valid) mh = max(mh, int(sv[h2 * 64 + t]));
          mx[h2] = mh;
        }
      }
      if (mx[0] != INT_MIN) m = fmaxf(m, fmaf(float(mx[0]), sc0, -kFp8Offset));
      if (mx[1] != INT_MIN) m = fmaxf(m, fmaf(float(mx[1]), sc1, -kFp8Offset));
    }
    // ---- P pass: P = 2^(s - m) per 64-key half -> E4M3 into TMEM
    float ds[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    uint64_t ds01 = f2_pack(0.0f, 0.0f), ds23 = f2_pack(0.0f, 0.0f);   // ds[0..3] as lane pairs
    float ks_cur = __ldg(ks_head);
    for (int i = 0; i < nh && ok; ++i) {
      const int h = i & 1;
      const float sc = qsl * ks_cur;          // one K scale block per half
      ks_cur = __ldg(ks_head + (i + 1 < nh ? i + 1 : 0));
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&sb_full[h]), (i >> 1) & 1, err))) { ok = false; break; }
      tc_fence_after();
      const int valid = kv_lim - i * kHalf;
      uint32_t sv[64];
      tc_ld_32x32b_x32(tmem + t_lane + uint32_t(h * kHalf), *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tc_ld_32x32b_x32(tmem + t_lane + uint32_t(h * kHalf + 32), *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tc_wait_ld();
      uint32_t w[16];
      p_half(sv, valid, sc, m, ds01, ds23, ds, w);
      tc_st_32x32b_x16(tmem + t_lane + uint32_t(h * kHalf), w);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&pb_full[h]));
    }
    {
      float d0, d1, d2, d3;
      f2_unpack(ds01, d0, d1);
      f2_unpack(ds23, d2, d3);
      ds[0] += d0;
      ds[1] += d1;
      ds[2] += d2;
      ds[3] += d3;
    }
    const float dsum = (ds[0] + ds[1]) + (ds[2] + ds[3]);
    if (ok && __all_sync(0xffffffffu, mbar_wait(smem_u32(o_full), 0, err))) {
      tc_fence_after();
      attn_store_row(p, tmem, t_lane, kTmemO, bh, q_tok, dsum);
    }
  }

  if (p.signal_peers) __threadfence_system();   // this CTA's peer stores before its signals
  tc_fence_before();
  __syncthreads();
  if (p.signal_peers && int(threadIdx.x) < p.peer_count)
    atomicAdd_system(p.signal_peers[threadIdx.x] + p.peer_slot, 1ull);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int make_rows_tmap(CUtensorMap* map, const void* base, int64_t rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(kD), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(kD)};
  cuuint32_t box[2] = {128u, 128u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return QIA_OK;
}

int64_t pad128(int64_t s) { return (s + 127) / 128 * 128; }

struct Workspace {
  int8_t* q8;
  int8_t* k8;
  uint8_t* v8;
  float* q_scale;
  float* k_scale;
  float* v_scale;
  __nv_bfloat16* k_mean;
  float* v_recp;
  float* k_part;   // [B*H, S_kv_pad/32, 128] per-32-row-tile K column sums
  float* v_part;   // [B*H, S_kv_pad/32, 128] per-32-row-tile |V| column maxima
  __nv_bfloat16* kn;  // [B*H, S_kv_pad, 128] normalised K (joint-sequence entry points)
};

int64_t workspace_layout(int64_t B, int64_t H, int64_t Sq, int64_t Skv, uint8_t* base, Workspace* ws) {
  const int64_t bh = B * H, sqp = pad128(Sq), skp = pad128(Skv);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = off;
    off += (bytes + 255) / 256 * 256;
    return base ? base + at : nullptr;
  };
  uint8_t* q8 = take(bh * sqp * kD);
  uint8_t* k8 = take(bh * skp * kD);
  uint8_t* v8 = take(bh * skp * kD);
  uint8_t* qs = take(bh * (sqp / 32) * 4);
  uint8_t* ks = take(bh * (skp / 64) * 4);
  uint8_t* vs = take(bh * kD * 4);
  uint8_t* km = take(bh * kD * 2);
  uint8_t* vr = take(bh * kD * 4);
  uint8_t* kpart = take(bh * (skp / 32) * kD * 4);
  uint8_t* vpart = take(bh * (skp / 32) * kD * 4);
  uint8_t* kn = take(bh * skp * kD * 2);
  if (ws) {
    ws->q8 = (int8_t*)q8;
    ws->k8 = (int8_t*)k8;
    ws->v8 = v8;
    ws->q_scale = (float*)qs;
    ws->k_scale = (float*)ks;
    ws->v_scale = (float*)vs;
    ws->k_mean = (__nv_bfloat16*)km;
    ws->v_recp = (float*)vr;
    ws->k_part = (float*)kpart;
    ws->v_part = (float*)vpart;
    ws->kn = (__nv_bfloat16*)kn;
  }
  return off;
}

struct Strides {
  int64_t b, s, h;
};

int check_nhd(const void* t, const Strides& st, const char* who) {
  if (!t) return set_error(QIA_ERR_INVALID, "%s: null tensor", who);
  if (!aligned(t, 16) || st.b % 8 || st.s % 8 || st.h % 8)
    return set_error(QIA_ERR_ALIGNMENT, "%s: tensors and strides must be 16-byte aligned", who);
  return QIA_OK;
}

// Opt the staged quantizer kernels of one source type into their dynamic
// shared memory, once per device.
template <class Src>
int quant_smem_attrs() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return QIA_OK;
  cudaError_t e = cudaFuncSetAttribute(sage_quant_q_stats_kernel<Src>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       q_stats_smem<Src>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(sage_quant_kv_kernel<Src>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmem);
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return QIA_OK;
}

template <class Src>
int quant_rows(const Src& src, int64_t B, int64_t H, int64_t Sq, int64_t Skv, const Workspace& ws, cudaStream_t st) {
  int rc = quant_smem_attrs<Src>();
  if (rc) return rc;
  const int64_t sqp = pad128(Sq), skp = pad128(Skv);
  const unsigned bh = unsigned(B * H), q_tiles = unsigned(sqp / kQBlock);
  const unsigned kv_tiles = unsigned((Skv + kQBlock - 1) / kQBlock);
  const int part_stride = int(skp / kQBlock);
  sage_quant_q_stats_kernel<Src><<<dim3(bh, q_tiles > kv_tiles ? q_tiles : kv_tiles), 256, q_stats_smem<Src>(), st>>>(
      src, int(Sq), int(sqp), int(Skv), int(H), int(kv_tiles), part_stride, ws.q8, ws.q_scale, ws.k_part, ws.v_part);
  rc = check_launch("sage_quant_q_stats_kernel");
  if (rc) return rc;
  sage_quant_finalize_kernel<<<dim3(bh, kD / 32), 256, 0, st>>>(ws.k_part, ws.v_part, int(kv_tiles), part_stride, int(Skv), ws.k_mean,
                                                 ws.v_scale, ws.v_recp);
  rc = check_launch("sage_quant_finalize_kernel");
  if (rc) return rc;
  sage_quant_kv_kernel<Src><<<dim3(bh, unsigned(skp / kQTile), 2), 256, kKvSmem, st>>>(
      src, int(Skv), int(skp), int(H), ws.k_mean, ws.v_recp, ws.k8, ws.k_scale, ws.v8);
  return check_launch("sage_quant_kv_kernel");
}

int quant_qkv(const void* q, Strides qs, const void* k, Strides ks, const void* v, Strides vs, int64_t B, int64_t H,
              int64_t Sq, int64_t Skv, const Workspace& ws, cudaStream_t st) {
  PlainQKV src;
  src.x[0] = (const __nv_bfloat16*)q;
  src.x[1] = (const __nv_bfloat16*)k;
  src.x[2] = (const __nv_bfloat16*)v;
  const Strides all[3] = {qs, ks, vs};
  for (int c = 0; c < 3; ++c) {
    src.sb[c] = all[c].b;
    src.ss[c] = all[c].s;
    src.sh[c] = all[c].h;
  }
  src.eps = 0.0f;
  return quant_rows(src, B, H, Sq, Skv, ws, st);
}

struct MxOut {
  void* a_values = nullptr;
  void* a_scales = nullptr;
  void* b_values = nullptr;
  void* b_scales = nullptr;
};

struct PeerOut {
  void* const* img = nullptr;
  void* const* txt = nullptr;
  void* const* signal = nullptr;
  int count = 0, rows = 0, head0 = 0, slot = 0;
  int64_t ld = 0;
};

int launch_attn(const Workspace& ws, void* out, Strides os, void* out2, Strides os2, int64_t split, int64_t B,
                int64_t H, int64_t Sq, int64_t Skv, float sm_scale, cudaStream_t st, const MxOut& mx = MxOut(),
                const int* kv_limit = nullptr, int64_t kv_limit_stride_b = 0, const PeerOut& peers = PeerOut()) {
  static bool attr_done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(sage_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
      if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_done[dev] = true;
    }
  }
  const int64_t sqp = pad128(Sq), skp = pad128(Skv);
  CUtensorMap tq, tk, tv;
  int rc = make_rows_tmap(&tq, ws.q8, B * H * sqp);
  if (rc) return rc;
  rc = make_rows_tmap(&tk, ws.k8, B * H * skp);
  if (rc) return rc;
  rc = make_rows_tmap(&tv, ws.v8, B * H * skp);
  if (rc) return rc;
  AttnParams p;
  p.q_scale = ws.q_scale;
  p.k_scale = ws.k_scale;
  p.v_scale = ws.v_scale;
  p.out = (__nv_bfloat16*)out;
  p.out_stride_b = os.b;
  p.out_stride_s = os.s;
  p.out_stride_h = os.h;
  p.out2 = (__nv_bfloat16*)out2;
  p.out2_stride_b = os2.b;
  p.out2_stride_s = os2.s;
  p.out2_stride_h = os2.h;
  p.split = (out2 || mx.a_values || peers.img) ? int(split) : int(Sq);
  p.B = int(B);
  p.H = int(H);
  p.Sq = int(Sq);
  p.Skv = int(Skv);
  p.Sq_pad = int(sqp);
  p.Skv_pad = int(skp);
  p.sm_scale_log2 = sm_scale * 1.44269504088896340736f;
  p.qa_values = (uint8_t*)mx.a_values;
  p.qa_scales = (uint8_t*)mx.a_scales;
  p.qb_values = (uint8_t*)mx.b_values;
  p.qb_scales = (uint8_t*)mx.b_scales;
  p.kv_limit = kv_limit;
  p.kv_limit_stride_b = kv_limit_stride_b;
  p.img_peers = (__nv_bfloat16* const*)peers.img;
  p.txt_peers = (__nv_bfloat16* const*)peers.txt;
  p.signal_peers = (unsigned long long* const*)peers.signal;
  p.peer_count = peers.count;
  p.peer_rows = peers.rows;
  p.peer_head0 = peers.head0;
  p.peer_slot = peers.slot;
  p.peer_ld = peers.ld;
  const dim3 grid = kv_limit ? dim3(unsigned(B * H), unsigned(sqp / 128)) : dim3(unsigned(sqp / 128), unsigned(B * H));
  sage_attn_kernel<<<grid, 192, kAttnSmem, st>>>(tq, tk, tv, p, device_error_word());
  return check_launch("sage_attn_kernel");
}

int check_sizes(int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t D, const char* who) {
  if (B <= 0 || H <= 0 || Sq <= 0 || Skv <= 0) return set_error(QIA_ERR_INVALID, "%s: bad sizes", who);
  if (D != kD) return set_error(QIA_ERR_UNSUPPORTED, "%s: head_dim must be 128", who);
  if (B * H > 65535 || pad128(Sq) * B * H > (1LL << 31) || pad128(Skv) * B * H > (1LL << 31))
    return set_error(QIA_ERR_UNSUPPORTED, "%s: too large", who);
  return QIA_OK;
}

// The Q/K/V source of the joint [stream 0, stream 1] sequence read straight
// from the two streams' fused q|k|v projection outputs.
int make_joint(const void* qkv0, int64_t ld0, const void* qkv1, int64_t ld1, const void* wq0, const void* wk0,
               const void* wq1, const void* wk1, const void* freqs0, const void* freqs1, int64_t len0, int64_t len1,
               int64_t heads, float eps, JointQKV* src, const char* who) {
  if (!qkv0 || !qkv1 || !wq0 || !wk0 || !wq1 || !wk1 || !freqs0 || !freqs1)
    return set_error(QIA_ERR_INVALID, "%s: null pointer", who);
  if (len0 <= 0 || len1 <= 0) return set_error(QIA_ERR_INVALID, "%s: stream lengths must be positive", who);
  if (ld0 < 3 * heads * kD || ld1 < 3 * heads * kD || ld0 % 8 || ld1 % 8)
    return set_error(QIA_ERR_INVALID, "%s: leading dimensions must be >= 3*heads*128 and multiples of 8", who);
  const void* ptrs[8] = {qkv0, qkv1, wq0, wk0, wq1, wk1, freqs0, freqs1};
  for (const void* p : ptrs)
    if (!aligned(p, 16)) return set_error(QIA_ERR_ALIGNMENT, "%s: 16-byte alignment", who);
  src->qkv0 = (const __nv_bfloat16*)qkv0;
  src->qkv1 = (const __nv_bfloat16*)qkv1;
  src->ld0 = ld0;
  src->ld1 = ld1;
  src->wq0 = (const __nv_bfloat16*)wq0;
  src->wk0 = (const __nv_bfloat16*)wk0;
  src->wq1 = (const __nv_bfloat16*)wq1;
  src->wk1 = (const __nv_bfloat16*)wk1;
  src->f0 = (const float*)freqs0;
  src->f1 = (const float*)freqs1;
  src->len0 = int(len0);
  src->len1 = int(len1);
  src->H = int(heads);
  src->eps = eps;
  src->kn = nullptr;
  src->S_pad = 0;
  return QIA_OK;
}

// ------------------------------------------------------------------ built-in scratch
// Scratch for qia_sage_attention_noalloc: a fixed device array that lives as
// long as the library is loaded (every GPU that loads the library holds these
// 16 MiB until the process exits). Host code must not use the symbol as a
// pointer: its device address is resolved per device by builtin_scratch().
constexpr int64_t kBuiltinScratchBytes = int64_t(16) << 20;
static __device__ __align__(256) uint8_t g_sage_scratch[kBuiltinScratchBytes];

// Device address of g_sage_scratch on the current device, looked up with
// cudaGetSymbolAddress the first time each device asks and cached after that.
int builtin_scratch(void** out) {
  static void* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(QIA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sage_scratch);
    if (e != cudaSuccess || !p)
      return set_error(QIA_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return QIA_OK;
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int64_t qia_sage_workspace_bytes(int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_kv) {
  if (batch <= 0 || heads <= 0 || seq_q <= 0 || seq_kv <= 0) return -1;
  return workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
}

extern "C" int qia_sage_attention(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                  int64_t seq_q, int64_t seq_kv, int64_t heads, int64_t head_dim,
                                  const int64_t* strides, float sm_scale, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attention");
  if (rc) return rc;
  if (!strides) return set_error(QIA_ERR_INVALID, "qia_sage_attention: null strides");
  const Strides sq{strides[0], strides[1], strides[2]}, sk{strides[3], strides[4], strides[5]},
      sv{strides[6], strides[7], strides[8]}, so{strides[9], strides[10], strides[11]};
  if ((rc = check_nhd(q, sq, "qia_sage_attention q")) || (rc = check_nhd(k, sk, "qia_sage_attention k")) ||
      (rc = check_nhd(v, sv, "qia_sage_attention v")) || (rc = check_nhd(out, so, "qia_sage_attention out")))
    return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return set_error(QIA_ERR_INVALID, "qia_sage_attention: workspace of %lld bytes needed", (long long)need);
  if (!aligned(workspace, 256)) return set_error(QIA_ERR_ALIGNMENT, "qia_sage_attention: workspace alignment 256");
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)workspace, &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  cudaStream_t st = as_stream(stream);
  rc = quant_qkv(q, sq, k, sk, v, sv, batch, heads, seq_q, seq_kv, ws, st);
  if (rc) return rc;
  return launch_attn(ws, out, so, nullptr, so, 0, batch, heads, seq_q, seq_kv, scale, st);
}

extern "C" int qia_sage_attention_prefill(const void* q, const void* k, const void* v, void* out,
                                          const int32_t* kv_limit, int64_t kv_limit_stride_b, int64_t batch,
                                          int64_t seq_q, int64_t seq_kv, int64_t heads, int64_t head_dim,
                                          const int64_t* strides, float sm_scale, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attention_prefill");
  if (rc) return rc;
  if (!strides) return set_error(QIA_ERR_INVALID, "qia_sage_attention_prefill: null strides");
  if (!kv_limit) return set_error(QIA_ERR_INVALID, "qia_sage_attention_prefill: null kv_limit");
  if (kv_limit_stride_b < 0 || (batch > 1 && kv_limit_stride_b != 0 && kv_limit_stride_b < seq_q))
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_prefill: kv_limit_stride_b must be 0 or >= seq_q");
  if (!aligned(kv_limit, 4)) return set_error(QIA_ERR_ALIGNMENT, "qia_sage_attention_prefill: kv_limit alignment 4");
  if (pad128(seq_q) / 128 > 65535) return set_error(QIA_ERR_UNSUPPORTED, "qia_sage_attention_prefill: seq_q too large");
  const Strides sq{strides[0], strides[1], strides[2]}, sk{strides[3], strides[4], strides[5]},
      sv{strides[6], strides[7], strides[8]}, so{strides[9], strides[10], strides[11]};
  if ((rc = check_nhd(q, sq, "qia_sage_attention_prefill q")) ||
      (rc = check_nhd(k, sk, "qia_sage_attention_prefill k")) ||
      (rc = check_nhd(v, sv, "qia_sage_attention_prefill v")) ||
      (rc = check_nhd(out, so, "qia_sage_attention_prefill out")))
    return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_prefill: workspace of %lld bytes needed", (long long)need);
  if (!aligned(workspace, 256))
    return set_error(QIA_ERR_ALIGNMENT, "qia_sage_attention_prefill: workspace alignment 256");
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)workspace, &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  cudaStream_t st = as_stream(stream);
  rc = quant_qkv(q, sq, k, sk, v, sv, batch, heads, seq_q, seq_kv, ws, st);
  if (rc) return rc;
  return launch_attn(ws, out, so, nullptr, so, 0, batch, heads, seq_q, seq_kv, scale, st, MxOut(), kv_limit,
                     kv_limit_stride_b);
}

extern "C" int qia_sage_attention_split(const void* q, const void* k, const void* v, void* out_a, void* out_b,
                                        int64_t split, int64_t batch, int64_t seq_q, int64_t seq_kv, int64_t heads,
                                        int64_t head_dim, const int64_t* strides, float sm_scale, void* workspace,
                                        int64_t workspace_bytes, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attention_split");
  if (rc) return rc;
  if (!strides) return set_error(QIA_ERR_INVALID, "qia_sage_attention_split: null strides");
  if (split <= 0 || split >= seq_q) return set_error(QIA_ERR_INVALID, "qia_sage_attention_split: 0 < split < seq_q");
  const Strides sq{strides[0], strides[1], strides[2]}, sk{strides[3], strides[4], strides[5]},
      sv{strides[6], strides[7], strides[8]}, sa{strides[9], strides[10], strides[11]},
      sb{strides[12], strides[13], strides[14]};
  if ((rc = check_nhd(q, sq, "qia_sage_attention_split q")) || (rc = check_nhd(k, sk, "qia_sage_attention_split k")) ||
      (rc = check_nhd(v, sv, "qia_sage_attention_split v")) ||
      (rc = check_nhd(out_a, sa, "qia_sage_attention_split out_a")) ||
      (rc = check_nhd(out_b, sb, "qia_sage_attention_split out_b")))
    return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_split: workspace of %lld bytes (256-aligned) needed",
                     (long long)need);
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)workspace, &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  cudaStream_t st = as_stream(stream);
  rc = quant_qkv(q, sq, k, sk, v, sv, batch, heads, seq_q, seq_kv, ws, st);
  if (rc) return rc;
  return launch_attn(ws, out_a, sa, out_b, sb, split, batch, heads, seq_q, seq_kv, scale, st);
}

extern "C" int qia_sage_attention_split_mx(const void* q, const void* k, const void* v, void* a_values,
                                           void* a_scales, void* b_values, void* b_scales, int64_t split,
                                           int64_t batch, int64_t seq_q, int64_t seq_kv, int64_t heads,
                                           int64_t head_dim, const int64_t* strides, float sm_scale, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attention_split_mx");
  if (rc) return rc;
  if (!strides) return set_error(QIA_ERR_INVALID, "qia_sage_attention_split_mx: null strides");
  // split == seq_q: one stream (every query token goes to a_*; b_* unused)
  if (split <= 0 || split > seq_q)
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_split_mx: 0 < split <= seq_q");
  const bool two = split < seq_q;
  if (!a_values || !a_scales || (two && (!b_values || !b_scales)))
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_split_mx: null output");
  if (!aligned(a_values, 32) || !aligned(a_scales, 4) || (two && (!aligned(b_values, 32) || !aligned(b_scales, 4))))
    return set_error(QIA_ERR_ALIGNMENT, "qia_sage_attention_split_mx: values 32-byte, scales 4-byte aligned");
  const Strides sq{strides[0], strides[1], strides[2]}, sk{strides[3], strides[4], strides[5]},
      sv{strides[6], strides[7], strides[8]};
  if ((rc = check_nhd(q, sq, "qia_sage_attention_split_mx q")) ||
      (rc = check_nhd(k, sk, "qia_sage_attention_split_mx k")) ||
      (rc = check_nhd(v, sv, "qia_sage_attention_split_mx v")))
    return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_split_mx: workspace of %lld bytes (256-aligned) needed",
                     (long long)need);
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)workspace, &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  cudaStream_t st = as_stream(stream);
  rc = quant_qkv(q, sq, k, sk, v, sv, batch, heads, seq_q, seq_kv, ws, st);
  if (rc) return rc;
  MxOut mx;
  mx.a_values = a_values;
  mx.a_scales = a_scales;
  mx.b_values = b_values;
  mx.b_scales = b_scales;
  const Strides none{0, 0, 0};
  return launch_attn(ws, nullptr, none, nullptr, none, split, batch, heads, seq_q, seq_kv, scale, st, mx);
}

extern "C" int qia_sage_quantize(const void* q, const void* k, const void* v, int64_t batch, int64_t seq_q,
                                 int64_t seq_kv, int64_t heads, int64_t head_dim, const int64_t* strides,
                                 void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_quantize");
  if (rc) return rc;
  if (!strides) return set_error(QIA_ERR_INVALID, "qia_sage_quantize: null strides");
  const Strides sq{strides[0], strides[1], strides[2]}, sk{strides[3], strides[4], strides[5]},
      sv{strides[6], strides[7], strides[8]};
  if ((rc = check_nhd(q, sq, "qia_sage_quantize q")) || (rc = check_nhd(k, sk, "qia_sage_quantize k")) ||
      (rc = check_nhd(v, sv, "qia_sage_quantize v")))
    return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return set_error(QIA_ERR_INVALID, "qia_sage_quantize: workspace of %lld bytes (256-aligned) needed",
                     (long long)need);
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)workspace, &ws);
  return quant_qkv(q, sq, k, sk, v, sv, batch, heads, seq_q, seq_kv, ws, as_stream(stream));
}

extern "C" int qia_sage_quantize_joint(const void* qkv0, int64_t ld0, const void* qkv1, int64_t ld1,
                                       const void* weight_q0, const void* weight_k0, const void* weight_q1,
                                       const void* weight_k1, const void* freqs0, const void* freqs1, int64_t batch,
                                       int64_t len0, int64_t len1, int64_t heads, int64_t head_dim, float eps,
                                       void* workspace, int64_t workspace_bytes, void* stream) {
  const int64_t S = len0 + len1;
  int rc = check_sizes(batch, heads, S, S, head_dim, "qia_sage_quantize_joint");
  if (rc) return rc;
  JointQKV src;
  rc = make_joint(qkv0, ld0, qkv1, ld1, weight_q0, weight_k0, weight_q1, weight_k1, freqs0, freqs1, len0, len1, heads,
                  eps, &src, "qia_sage_quantize_joint");
  if (rc) return rc;
  const int64_t need = workspace_layout(batch, heads, S, S, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return set_error(QIA_ERR_INVALID, "qia_sage_quantize_joint: workspace of %lld bytes (256-aligned) needed",
                     (long long)need);
  Workspace ws;
  workspace_layout(batch, heads, S, S, (uint8_t*)workspace, &ws);
  src.kn = ws.kn;
  src.S_pad = int(pad128(S));
  return quant_rows(src, batch, heads, S, S, ws, as_stream(stream));
}

extern "C" int qia_sage_attention_joint_mx(const void* qkv0, int64_t ld0, const void* qkv1, int64_t ld1,
                                           const void* weight_q0, const void* weight_k0, const void* weight_q1,
                                           const void* weight_k1, const void* freqs0, const void* freqs1,
                                           void* a_values, void* a_scales, void* b_values, void* b_scales,
                                           int64_t batch, int64_t len0, int64_t len1, int64_t heads,
                                           int64_t head_dim, float eps, float sm_scale, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  const int64_t S = len0 + len1;
  int rc = check_sizes(batch, heads, S, S, head_dim, "qia_sage_attention_joint_mx");
  if (rc) return rc;
  if (!a_values || !a_scales || !b_values || !b_scales)
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_joint_mx: null output");
  if (!aligned(a_values, 32) || !aligned(b_values, 32) || !aligned(a_scales, 4) || !aligned(b_scales, 4))
    return set_error(QIA_ERR_ALIGNMENT, "qia_sage_attention_joint_mx: values 32-byte, scales 4-byte aligned");
  JointQKV src;
  rc = make_joint(qkv0, ld0, qkv1, ld1, weight_q0, weight_k0, weight_q1, weight_k1, freqs0, freqs1, len0, len1, heads,
                  eps, &src, "qia_sage_attention_joint_mx");
  if (rc) return rc;
  const int64_t need = workspace_layout(batch, heads, S, S, nullptr, nullptr);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return set_error(QIA_ERR_INVALID, "qia_sage_attention_joint_mx: workspace of %lld bytes (256-aligned) needed",
                     (long long)need);
  Workspace ws;
  workspace_layout(batch, heads, S, S, (uint8_t*)workspace, &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  cudaStream_t st = as_stream(stream);
  src.kn = ws.kn;
  src.S_pad = int(pad128(S));
  rc = quant_rows(src, batch, heads, S, S, ws, st);
  if (rc) return rc;
  MxOut mx;
  mx.a_values = a_values;
  mx.a_scales = a_scales;
  mx.b_values = b_values;
  mx.b_scales = b_scales;
  const Strides none{0, 0, 0};
  return launch_attn(ws, nullptr, none, nullptr, none, len0, batch, heads, S, S, scale, st, mx);
}

extern "C" int qia_sage_attn_quantized(const void* workspace, void* out, int64_t batch, int64_t seq_q,
                                       int64_t seq_kv, int64_t heads, int64_t head_dim, const int64_t* out_strides,
                                       float sm_scale, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attn_quantized");
  if (rc) return rc;
  if (!workspace || !aligned(workspace, 256) || !out_strides)
    return set_error(QIA_ERR_INVALID, "qia_sage_attn_quantized: workspace/out_strides");
  const Strides so{out_strides[0], out_strides[1], out_strides[2]};
  if ((rc = check_nhd(out, so, "qia_sage_attn_quantized out"))) return rc;
  Workspace ws;
  workspace_layout(batch, heads, seq_q, seq_kv, (uint8_t*)const_cast<void*>(workspace), &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  return launch_attn(ws, out, so, nullptr, so, 0, batch, heads, seq_q, seq_kv, scale, as_stream(stream));
}

extern "C" int64_t qia_sage_attn_ctas(int64_t batch, int64_t heads, int64_t seq_q) {
  if (batch <= 0 || heads <= 0 || seq_q <= 0) return -1;
  return batch * heads * (pad128(seq_q) / 128);
}

extern "C" int qia_sage_attn_quantized_peers(const void* workspace, int64_t seq, int64_t heads, int64_t head_dim,
                                             int64_t split, void* const* img_peers, void* const* txt_peers,
                                             int64_t peer_rows, int64_t peer_count, int64_t head0,
                                             int64_t heads_total, void* const* signal_peers, int64_t slot,
                                             float sm_scale, void* stream) {
  int rc = check_sizes(1, heads, seq, seq, head_dim, "qia_sage_attn_quantized_peers");
  if (rc) return rc;
  if (!workspace || !aligned(workspace, 256) || !img_peers || !txt_peers || !signal_peers)
    return set_error(QIA_ERR_INVALID, "qia_sage_attn_quantized_peers: null pointer");
  if (peer_count <= 0 || peer_count > 64 || slot < 0 || slot >= peer_count || split <= 0 || split >= seq ||
      peer_rows <= 0 || (seq - split) != peer_rows * peer_count || head0 < 0 || head0 + heads > heads_total)
    return set_error(QIA_ERR_INVALID,
                     "qia_sage_attn_quantized_peers: seq=%lld split=%lld rows=%lld ranks=%lld heads %lld+%lld of %lld",
                     (long long)seq, (long long)split, (long long)peer_rows, (long long)peer_count, (long long)head0,
                     (long long)heads, (long long)heads_total);
  Workspace ws;
  workspace_layout(1, heads, seq, seq, (uint8_t*)const_cast<void*>(workspace), &ws);
  const float scale = sm_scale > 0.0f ? sm_scale : 1.0f / sqrtf(float(head_dim));
  PeerOut po;
  po.img = img_peers;
  po.txt = txt_peers;
  po.signal = signal_peers;
  po.count = int(peer_count);
  po.rows = int(peer_rows);
  po.head0 = int(head0);
  po.slot = int(slot);
  po.ld = heads_total * kD;
  const Strides none{0, 0, 0};
  return launch_attn(ws, nullptr, none, nullptr, none, split, 1, heads, seq, seq, scale, as_stream(stream), MxOut(),
                     nullptr, 0, po);
}

// Same computation as qia_sage_attention, with the library's built-in scratch
// in place of a caller workspace, for callers that cannot allocate device
// memory (see qia_b200.h). Every region of the scratch is rewritten before it
// is read on each call, so nothing needs clearing between calls; calls that
// overlap on the GPU (other streams, other host threads) share the one array
// and race.
extern "C" int qia_sage_attention_noalloc(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                          int64_t seq_q, int64_t seq_kv, int64_t heads, int64_t head_dim,
                                          const int64_t* strides, float sm_scale, void* stream) {
  int rc = check_sizes(batch, heads, seq_q, seq_kv, head_dim, "qia_sage_attention_noalloc");
  if (rc) return rc;
  const int64_t need = workspace_layout(batch, heads, seq_q, seq_kv, nullptr, nullptr);
  if (need > kBuiltinScratchBytes)
    return set_error(QIA_ERR_UNSUPPORTED,
                     "qia_sage_attention_noalloc: these sizes need %lld bytes of scratch but the built-in scratch "
                     "holds %lld; use qia_sage_attention with a caller workspace",
                     (long long)need, (long long)kBuiltinScratchBytes);
  void* ws = nullptr;
  rc = builtin_scratch(&ws);
  if (rc) return rc;
  return qia_sage_attention(q, k, v, out, batch, seq_q, seq_kv, heads, head_dim, strides, sm_scale, ws,
                            kBuiltinScratchBytes, stream);
}
