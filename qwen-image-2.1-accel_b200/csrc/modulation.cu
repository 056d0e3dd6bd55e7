// AdaLN modulation vectors of one dual-stream block: y = W . x + b for the
// block's stacked img_mod/txt_mod linears (W: [12 * unit, K] bf16, the two
// streams' six chunks of width `unit` each), with the two scale chunks of
// every six returned as 1 + scale (bf16 rounding after the linear and again
// after the +1, as the eager `1 + scale` on the bf16 linear output does).
//
// Reference: the v1 block's img_mod / txt_mod Linear(SiLU(temb)) and the
// (1 + scale) of _modulate (WHL:diffusers/models/transformers/
// transformer_qwenimage.py:683-717).
//
// Weight-read bound (K * 2 bytes per output). One warp per output row: the
// lanes read the row in 16-byte pieces (pieces lane, lane + 32, ...), multiply
// them with x held in shared memory, accumulate in fp32 in that order, then a
// xor-shuffle tree (16, 8, 4, 2, 1); lane 0 adds the bias in fp32 and rounds.
// The footprint is deliberately small (128 threads, K * 2 bytes of shared
// memory, few registers) so that a launch on a side stream runs on the SM
// resources the block's GEMM and attention leave free.
#include "qia_common.cuh"

namespace qia {
namespace {

constexpr int kModThreads = 128;

__global__ void __launch_bounds__(kModThreads) adaln_modulation_kernel(const __nv_bfloat16* __restrict__ x,
                                                                       const __nv_bfloat16* __restrict__ w,
                                                                       const __nv_bfloat16* __restrict__ b,
                                                                       __nv_bfloat16* __restrict__ y, int n, int k,
                                                                       int unit) {
  extern __shared__ __align__(16) uint4 s_x[];
  const int t = threadIdx.x, lane = t & 31;
  const int pieces = k / 8;
  for (int i = t; i < pieces; i += kModThreads) s_x[i] = __ldg(reinterpret_cast<const uint4*>(x) + i);
  __syncthreads();
  const int warps = gridDim.x * (kModThreads / 32);
  for (int row = blockIdx.x * (kModThreads / 32) + (t >> 5); row < n; row += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + int64_t(row) * k);
    float acc = 0.0f;
#pragma unroll 4
    for (int j = lane; j < pieces; j += 32) {
      float wf[8], xf[8];
      unpack8(__ldg(wr + j), wf);
      unpack8(s_x[j], xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = __fmaf_rn(wf[e], xf[e], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float v = round_bf16(__fadd_rn(acc, __bfloat162float(b[row])));
      const int chunk = (row / unit) % 6;
      if (chunk == 1 || chunk == 4) v = round_bf16(__fadd_rn(v, 1.0f));
      y[row] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_adaln_modulation(const void* x, const void* weight, const void* bias, void* out, int64_t n,
                                    int64_t k, int64_t unit, int64_t ctas, void* stream) {
  if (!x || !weight || !bias || !out) return set_error(QIA_ERR_INVALID, "qia_adaln_modulation: null pointer");
  if (n <= 0 || k <= 0 || unit <= 0 || n % (6 * unit) || ctas <= 0)
    return set_error(QIA_ERR_INVALID, "qia_adaln_modulation: n must be a positive multiple of 6 * unit, ctas > 0");
  if (k % 8 || k > 16384) return set_error(QIA_ERR_UNSUPPORTED, "qia_adaln_modulation: k must be a multiple of 8, <= 16384");
  if (n > (1LL << 30)) return set_error(QIA_ERR_UNSUPPORTED, "qia_adaln_modulation: n too large");
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(bias, 2) || !aligned(out, 2))
    return set_error(QIA_ERR_ALIGNMENT, "qia_adaln_modulation: x and weight must be 16-byte aligned");
  const int64_t max_ctas = (n + kModThreads / 32 - 1) / (kModThreads / 32);
  const unsigned grid = unsigned(ctas < max_ctas ? ctas : max_ctas);
  adaln_modulation_kernel<<<grid, kModThreads, size_t(k) * 2, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (const __nv_bfloat16*)bias, (__nv_bfloat16*)out,
      int(n), int(k), int(unit));
  return check_launch("adaln_modulation_kernel");
}
