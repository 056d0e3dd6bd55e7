// MXFP8 activation quantizer, SwiGLU (+ quantize) and GELU-tanh.
//
// Quantizer numerics (reference src/qwen_image_accel/kernels/mxfp8.py:31-56):
// per 1x32 block along K, E8M0 exponent from the fp32 bits of the block amax,
// codes = E4M3(x * 2^(127-e)) with round-to-nearest-even and saturation, and the
// scale byte stored in the 128x4 blocked layout. Rows past `rows` (padding up
// to a multiple of 128) quantize to zero codes and zero exponents.
//
// SwiGLU numerics (reference kernels/bf16.py:12-24): silu = div.rn(g, 1+exp(-g))
// rounded to bf16, times the value in fp32, rounded to bf16.
// GELU-tanh numerics: PyTorch's CUDA formula
// 0.5*x*(1 + tanh(sqrt(2/pi) * (x + 0.044715*x^3))) in fp32, rounded to bf16.
//
// Work split: 8 contiguous bf16 (one 16-byte load) per thread; a 32-element
// MX block is 4 adjacent lanes, its amax a 2-step xor tree inside the group.
#include "qia_common.cuh"

#include <math.h>

#include <mutex>

namespace qia {
namespace {



// Quantize 8 values (one quarter of an MX block) held by this lane; the 4 lanes
// of the block are adjacent and aligned (lane % 4 == 0 starts a block).
__device__ __forceinline__ void mx_quant8(const float (&y)[8], uint8_t* __restrict__ qv, uint8_t* __restrict__ qs,
                                          int64_t row, int64_t col, int64_t k) {
  const unsigned mask = 0xfu << (threadIdx.x & 28);
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
  amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
  const int e = mx_exponent(amax);
  const float inv = mx_inverse_scale(e);
  uint2 codes;
  codes.x = cvt_e4m3x4(y[0] * inv, y[1] * inv, y[2] * inv, y[3] * inv);
  codes.y = cvt_e4m3x4(y[4] * inv, y[5] * inv, y[6] * inv, y[7] * inv);
  *reinterpret_cast<uint2*>(qv + row * k + col) = codes;
  if ((col & 31) == 0) qs[mx_scale_offset(row, col >> 5, k >> 7)] = uint8_t(e);
}

__global__ void mx_quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, uint8_t* __restrict__ qv,
                                   uint8_t* __restrict__ qs, int64_t rows, int64_t k, int64_t n8) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t row = e / k, col = e - row * k;
    float y[8];
    if (row < rows) {
      unpack8(__ldg(reinterpret_cast<const uint4*>(x + row * ld + col)), y);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.0f;
    }
    mx_quant8(y, qv, qs, row, col, k);
  }
}

__global__ void swiglu_kernel(const uint4* __restrict__ g, const uint4* __restrict__ v, uint4* __restrict__ out,
                              int64_t n8) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    float fg[8], fv[8], o[8];
    unpack8(__ldg(g + i), fg);
    unpack8(__ldg(v + i), fv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(silu_ref(fg[j]), fv[j]);
    out[i] = pack8(o);
  }
}

__global__ void swiglu_quant_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ v,
                                    uint8_t* __restrict__ qv, uint8_t* __restrict__ qs, int64_t rows, int64_t k,
                                    int64_t n8) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t row = e / k, col = e - row * k;
    float y[8];
    if (row < rows) {
      float fg[8], fv[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(g + e)), fg);
      unpack8(__ldg(reinterpret_cast<const uint4*>(v + e)), fv);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = round_bf16(__fmul_rn(silu_ref(fg[j]), fv[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.0f;
    }
    mx_quant8(y, qv, qs, row, col, k);
  }
}

// SwiGLU + quantizer for large inputs: the gate is bf16, so silu(g) takes one
// of 65,536 values. Each CTA first tabulates silu_ref over every bf16 bit
// pattern in shared memory (128 KB, the same device function, so every entry
// is exactly what the direct kernel computes) and then looks it up, which
// leaves the kernel bound by HBM instead of by the IEEE divide and exp of
// every element. Two 16-byte loads of gate and value per thread are in flight
// per trip.
constexpr int kSiluTableThreads = 1024;
constexpr int kSiluTableBytes = 65536 * 2;

__device__ __forceinline__ void swiglu_table8(const uint4& g, const uint4& v, const uint16_t* __restrict__ tab,
                                              float (&y)[8]) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
  float fv[8];
  unpack8(v, fv);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float s0 = __uint_as_float(uint32_t(tab[gw[m] & 0xffffu]) << 16);
    const float s1 = __uint_as_float(uint32_t(tab[gw[m] >> 16]) << 16);
    y[2 * m] = round_bf16(__fmul_rn(s0, fv[2 * m]));
    y[2 * m + 1] = round_bf16(__fmul_rn(s1, fv[2 * m + 1]));
  }
}

__global__ void __launch_bounds__(kSiluTableThreads, 1)
swiglu_quant_table_kernel(const uint4* __restrict__ g, const uint4* __restrict__ v, uint8_t* __restrict__ qv,
                          uint8_t* __restrict__ qs, int64_t rows, int64_t k, int64_t n8) {
  extern __shared__ uint16_t silu_tab[];
  for (int i = threadIdx.x; i < 65536; i += blockDim.x)
    silu_tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(silu_ref(__uint_as_float(uint32_t(i) << 16))));
  __syncthreads();
  // rows past `rows` (the padding up to 128) read as zero gate and value:
  // bf16(silu(0) * 0) = 0, the zero codes the direct kernel writes
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += 2 * stride) {
    const int64_t i2 = i + stride;
    const bool has2 = i2 < n8;                  // uniform in each aligned 4-lane MX group
    const int64_t row0 = (i * 8) / k, row1 = (i2 * 8) / k;
    const bool live0 = row0 < rows, live1 = has2 && row1 < rows;
    const uint4 g0 = live0 ? __ldg(g + i) : zero, v0 = live0 ? __ldg(v + i) : zero;
    const uint4 g1 = live1 ? __ldg(g + i2) : zero, v1 = live1 ? __ldg(v + i2) : zero;
    float y[8];
    swiglu_table8(g0, v0, silu_tab, y);
    mx_quant8(y, qv, qs, row0, i * 8 - row0 * k, k);
    if (has2) {
      swiglu_table8(g1, v1, silu_tab, y);
      mx_quant8(y, qv, qs, row1, i2 * 8 - row1 * k, k);
    }
  }
}

__global__ void gelu_tanh_kernel(const uint4* __restrict__ x, uint4* __restrict__ out, int64_t n8) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    float f[8];
    unpack8(__ldg(x + i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = round_bf16(gelu_tanh_f32(f[j]));
    out[i] = pack8(f);
  }
}

unsigned flat_grid(int64_t n8, int threads) {
  int64_t blocks = (n8 + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return unsigned(blocks);
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_mxfp8_quantize(const void* x, int64_t ld, void* q_values, void* q_scales, int64_t rows,
                                  int64_t k, void* stream) {
  if (!x || !q_values || !q_scales) return set_error(QIA_ERR_INVALID, "qia_mxfp8_quantize: null pointer");
  if (rows <= 0 || k <= 0 || ld < k) return set_error(QIA_ERR_INVALID, "qia_mxfp8_quantize: bad sizes");
  if (k % 128 != 0) return set_error(QIA_ERR_UNSUPPORTED, "qia_mxfp8_quantize: k %% 128 != 0");
  if (ld % 8 != 0 || !aligned(x, 16) || !aligned(q_values, 16))
    return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_quantize: 16-byte alignment of x/ld/q_values");
  const int64_t padded = (rows + 127) / 128 * 128;
  const int64_t n8 = padded * k / 8;
  mx_quantize_kernel<<<flat_grid(n8, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, ld, (uint8_t*)q_values, (uint8_t*)q_scales, rows, k, n8);
  return check_launch("mx_quantize_kernel");
}

extern "C" int qia_swiglu(const void* gate, const void* value, void* out, int64_t n, void* stream) {
  if (!gate || !value || !out) return set_error(QIA_ERR_INVALID, "qia_swiglu: null pointer");
  if (n <= 0 || n % 8 != 0) return set_error(QIA_ERR_UNSUPPORTED, "qia_swiglu: n must be a positive multiple of 8");
  if (!aligned(gate, 16) || !aligned(value, 16) || !aligned(out, 16))
    return set_error(QIA_ERR_ALIGNMENT, "qia_swiglu: 16-byte alignment");
  swiglu_kernel<<<flat_grid(n / 8, 256), 256, 0, as_stream(stream)>>>((const uint4*)gate, (const uint4*)value,
                                                                       (uint4*)out, n / 8);
  return check_launch("swiglu_kernel");
}

extern "C" int qia_swiglu_quant(const void* gate, const void* value, void* q_values, void* q_scales, int64_t rows,
                                int64_t width, void* stream) {
  if (!gate || !value || !q_values || !q_scales) return set_error(QIA_ERR_INVALID, "qia_swiglu_quant: null pointer");
  if (rows <= 0 || width <= 0) return set_error(QIA_ERR_INVALID, "qia_swiglu_quant: bad sizes");
  if (width % 128 != 0) return set_error(QIA_ERR_UNSUPPORTED, "qia_swiglu_quant: width %% 128 != 0");
  if (!aligned(gate, 16) || !aligned(value, 16) || !aligned(q_values, 16))
    return set_error(QIA_ERR_ALIGNMENT, "qia_swiglu_quant: 16-byte alignment");
  const int64_t padded = (rows + 127) / 128 * 128;
  const int64_t n8 = padded * width / 8;
  // above ~8M elements the table's set-up (65,536 silu per CTA) is repaid
  if (n8 >= (int64_t(1) << 20)) {
    static bool attr_done[64] = {false};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(swiglu_quant_table_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSiluTableBytes);
        if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_done[dev] = true;
      }
    }
    int64_t blocks = (n8 + 2 * kSiluTableThreads - 1) / (2 * kSiluTableThreads);
    if (blocks > sm_count()) blocks = sm_count();
    swiglu_quant_table_kernel<<<unsigned(blocks), kSiluTableThreads, kSiluTableBytes, as_stream(stream)>>>(
        (const uint4*)gate, (const uint4*)value, (uint8_t*)q_values, (uint8_t*)q_scales, rows, width, n8);
    return check_launch("swiglu_quant_table_kernel");
  }
  swiglu_quant_kernel<<<flat_grid(n8, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)gate, (const __nv_bfloat16*)value, (uint8_t*)q_values, (uint8_t*)q_scales, rows, width,
      n8);
  return check_launch("swiglu_quant_kernel");
}

extern "C" int qia_gelu_tanh(const void* x, void* out, int64_t n, void* stream) {
  if (!x || !out) return set_error(QIA_ERR_INVALID, "qia_gelu_tanh: null pointer");
  if (n <= 0 || n % 8 != 0) return set_error(QIA_ERR_UNSUPPORTED, "qia_gelu_tanh: n must be a positive multiple of 8");
  if (!aligned(x, 16) || !aligned(out, 16)) return set_error(QIA_ERR_ALIGNMENT, "qia_gelu_tanh: 16-byte alignment");
  gelu_tanh_kernel<<<flat_grid(n / 8, 256), 256, 0, as_stream(stream)>>>((const uint4*)x, (uint4*)out, n / 8);
  return check_launch("gelu_tanh_kernel");
}
