// True-CFG combine with norm rescaling and the flow-match Euler update, one
// launch (reference: the v1 pipeline's CFG combine,
// WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681, and the
// Euler step x + (sigma_next - sigma) * v,
// WHL:diffusers/schedulers/scheduling_flow_match_euler_discrete.py:483-517).
//
// Per row (one token's velocity, dim channels), with every eager bf16 tensor
// boundary kept as a bf16 rounding:
//   comb  = bf16(neg + bf16(s * bf16(cond - neg)))
//   ratio = bf16(bf16(||cond||) / bf16(||comb||))        (fp32 sums of squares)
//   v     = bf16(comb * ratio)
//   out   = bf16(float(latent) + float(bf16(dt * v)))
// One warp per row; the sums of squares are a per-lane sum over the lane's
// channels (c = lane, lane + 32, ...) and a xor-shuffle tree. dt is a launch
// argument (qia_cfg_euler) or sigma_next - sigma from device memory
// (qia_cfg_euler_sched, so a captured step replays with each step's schedule).
#include "qia_common.cuh"

namespace qia {
namespace {

__global__ void __launch_bounds__(256) cfg_euler_kernel(const __nv_bfloat16* __restrict__ cond,
                                                        const __nv_bfloat16* __restrict__ neg,
                                                        const __nv_bfloat16* __restrict__ lat,
                                                        __nv_bfloat16* __restrict__ out, int64_t rows, int dim,
                                                        float s, float dt, const float* __restrict__ sigmas) {
  const int lane = threadIdx.x & 31;
  if (sigmas) dt = __fsub_rn(sigmas[1], sigmas[0]);   // the schedule's fp32 step, read on the device
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t base = row * dim;
    float ss_c = 0.0f, ss_m = 0.0f;
    for (int c = lane; c < dim; c += 32) {
      const float cv = __bfloat162float(cond[base + c]), nv = __bfloat162float(neg[base + c]);
      const float comb = round_bf16(__fadd_rn(nv, round_bf16(__fmul_rn(s, round_bf16(__fsub_rn(cv, nv))))));
      ss_c = __fmaf_rn(cv, cv, ss_c);
      ss_m = __fmaf_rn(comb, comb, ss_m);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss_c += __shfl_xor_sync(0xffffffffu, ss_c, o);
      ss_m += __shfl_xor_sync(0xffffffffu, ss_m, o);
    }
    const float ratio = round_bf16(__fdiv_rn(round_bf16(sqrtf(ss_c)), round_bf16(sqrtf(ss_m))));
    for (int c = lane; c < dim; c += 32) {
      const float cv = __bfloat162float(cond[base + c]), nv = __bfloat162float(neg[base + c]);
      const float comb = round_bf16(__fadd_rn(nv, round_bf16(__fmul_rn(s, round_bf16(__fsub_rn(cv, nv))))));
      const float v = round_bf16(__fmul_rn(comb, ratio));
      const float dv = round_bf16(__fmul_rn(dt, v));
      out[base + c] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(lat[base + c]), dv));
    }
  }
}

}  // namespace
}  // namespace qia

using namespace qia;

namespace {
int launch_cfg_euler(const void* cond, const void* neg, const void* latents, void* out, int64_t rows, int64_t dim,
                     float cfg_scale, float dt, const float* sigmas, void* stream, const char* name) {
  if (!cond || !neg || !latents || !out) return set_error(QIA_ERR_INVALID, "%s: null pointer", name);
  if (rows <= 0 || dim <= 0) return set_error(QIA_ERR_INVALID, "%s: rows=%lld dim=%lld", name,
                                              (long long)rows, (long long)dim);
  if (dim > 65536) return set_error(QIA_ERR_UNSUPPORTED, "%s: dim too large", name);
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  cfg_euler_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)cond, (const __nv_bfloat16*)neg, (const __nv_bfloat16*)latents, (__nv_bfloat16*)out,
      rows, int(dim), cfg_scale, dt, sigmas);
  return check_launch("cfg_euler_kernel");
}
}  // namespace

extern "C" int qia_cfg_euler(const void* cond, const void* neg, const void* latents, void* out, int64_t rows,
                             int64_t dim, float cfg_scale, float dt, void* stream) {
  return launch_cfg_euler(cond, neg, latents, out, rows, dim, cfg_scale, dt, nullptr, stream, "qia_cfg_euler");
}

extern "C" int qia_cfg_euler_sched(const void* cond, const void* neg, const void* latents, void* out, int64_t rows,
                                   int64_t dim, float cfg_scale, const void* sigmas, void* stream) {
  if (!sigmas) return set_error(QIA_ERR_INVALID, "qia_cfg_euler_sched: null sigmas");
  if (!aligned(sigmas, 4)) return set_error(QIA_ERR_ALIGNMENT, "qia_cfg_euler_sched: misaligned sigmas");
  return launch_cfg_euler(cond, neg, latents, out, rows, dim, cfg_scale, 0.0f, (const float*)sigmas, stream,
                          "qia_cfg_euler_sched");
}
