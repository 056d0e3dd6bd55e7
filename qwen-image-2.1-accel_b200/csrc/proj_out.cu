// The denoise step's tail in one tcgen05 kernel: proj_out (bf16 GEMM, bias)
// of both CFG rows, the true-CFG combine with norm rescaling and the
// flow-match Euler update, written straight into the new latents.
//
// Reference sequence (eager, one bf16 rounding at every tensor boundary):
//   v      = proj_out(y) = bf16(y @ W^T + b)        per CFG row (cond, uncond)
//            (WHL:diffusers/models/transformers/transformer_qwenimage.py:1007-1012)
//   comb   = bf16(neg + bf16(s * bf16(cond - neg)))
//   ratio  = bf16(bf16(||cond||) / bf16(||comb||))  (fp32 sums of squares)
//   v      = bf16(comb * ratio)
//            (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:666-671)
//   out    = bf16(float(latent) + float(bf16(dt * v))),  dt = sigma_next - sigma in fp32
//            (WHL:diffusers/schedulers/scheduling_flow_match_euler_discrete.py:483-517)
//
// Layout: y is the norm_out output of the CFG batch, bf16 [2 * rows, K]
// row-major (rows [0, rows) the conditional branch, [rows, 2 rows) the
// unconditional one, token for token); W bf16 [64, K]; latents / out bf16
// [rows, 64] (out may be latents). sigma and sigma_next are read from device
// memory, so a captured step replays with each step's schedule.
//
// One CTA per 64 tokens (192 threads): warp 0 issues the TMA loads (per K
// block of 64: the 64 tokens' cond rows into rows 0-63 of the A tile, their
// uncond rows into rows 64-127, and W), warp 1 the MMAs (M = 128, N = 64,
// K = 16 each, fp32 accumulator in 64 TMEM columns), warps 2-5 the epilogue:
// every thread owns one accumulator row; the uncond rows go to shared memory
// as bf16, and the 64 threads of the cond rows finish the combine and the
// Euler update for their tokens. Every wait is bounded (1 s) and reports
// QIA_ERR_TIMEOUT through the device error word.
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace qia {
namespace {

constexpr int kPoTok = 64;                       // tokens per CTA
constexpr int kPoK = 64;                         // K per stage: 128-byte rows, 128-byte swizzle
constexpr int kPoN = 64;                         // proj_out width (patch^2 x out_channels)
constexpr int kPoStages = 4;
constexpr int kPoABytes = 2 * kPoTok * kPoK * 2;  // cond + uncond rows: 16 KB
constexpr int kPoBBytes = kPoN * kPoK * 2;        // 8 KB
constexpr int kPoStageBytes = kPoABytes + kPoBBytes;
constexpr int kPoNegBytes = kPoTok * kPoN * 2;    // the uncond rows' proj_out values, bf16
constexpr int kPoSmem = kPoStages * kPoStageBytes + kPoNegBytes + 256 + 1024;
constexpr uint32_t kPoTmemCols = 64;
// kind::f16: f32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9, 10-12 = 1),
// both K-major, N = 64, M = 128
constexpr uint32_t kPoIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kPoN >> 3) << 17) |
                              (uint32_t(128 >> 4) << 24);

__device__ __forceinline__ void tc_mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

struct PoParams {
  const __nv_bfloat16* bias;   // [64] or null
  const __nv_bfloat16* lat;    // [rows, 64]
  __nv_bfloat16* out;          // [rows, 64]
  const float* sigmas;         // {sigma, sigma_next}
  int rows;
  int k_blocks;
  float s;                     // CFG scale
};

__global__ void __launch_bounds__(192, 2)
proj_out_cfg_euler_kernel(const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_w,
                          PoParams p, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* negs = reinterpret_cast<__nv_bfloat16*>(smem + kPoStages * kPoStageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPoStages * kPoStageBytes + kPoNegBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPoStages;
  uint64_t* acc_full = bars + 2 * kPoStages;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * kPoTok;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPoStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    mbar_init(smem_u32(drain), 1);
    fence_barrier_init();
    prefetch_tmap(&tm_y);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), kPoTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (!mbar_wait(smem_u32(&empty[s]), phase ^ 1, err)) { ok = false; break; }
        uint8_t* st = smem + s * kPoStageBytes;
        const uint32_t fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(fb, kPoStageBytes);
        tma_load_2d(smem_u32(st), &tm_y, fb, kb * kPoK, tok0);                       // cond rows
        tma_load_2d(smem_u32(st + kPoABytes / 2), &tm_y, fb, kb * kPoK, p.rows + tok0);  // uncond rows
        tma_load_2d(smem_u32(st + kPoABytes), &tm_w, fb, kb * kPoK, 0);
        ++issued;
        if (++s == kPoStages) { s = 0; phase ^= 1; }
      }
      if (!ok) {
        for (int i = 0; i < kPoStages && i < issued; ++i) {
          if (--s < 0) { s = kPoStages - 1; phase ^= 1; }
          mbar_wait(smem_u32(&full[s]), phase, nullptr, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t smem0 = smem_u32(smem);
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (!mbar_wait(smem_u32(&full[s]), phase, err)) { ok = false; break; }
        const uint64_t adesc = smem_desc_k_sw128(smem0 + uint32_t(s * kPoStageBytes));
        const uint64_t bdesc = smem_desc_k_sw128(smem0 + uint32_t(s * kPoStageBytes + kPoABytes));
#pragma unroll
        for (int j = 0; j < kPoK / 16; ++j)      // K = 16 per MMA: 32 bytes further along the row
          tc_mma_bf16(tmem_base, adesc + uint64_t(2 * j), bdesc + uint64_t(2 * j), kPoIdesc, (kb | j) != 0);
        tc_commit(smem_u32(&empty[s]));
        if (++s == kPoStages) { s = 0; phase ^= 1; }
      }
      if (ok) tc_commit(smem_u32(acc_full));
      tc_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, ok ? err : nullptr, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;                // TMEM sub-partition: accumulator rows 32 sub .. 32 sub + 31
    const int row = sub * 32 + lane;         // 0-63: cond of token tok0 + row; 64-127: uncond of tok0 + row - 64
    const bool got = __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_full), 0, err));
    float y[kPoN];
    if (got) {
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t t_row = tmem_base + (uint32_t(sub * 32) << 16);
      tc_ld_32x32b_x32(t_row, r0);
      tc_ld_32x32b_x32(t_row + 32u, r1);
      tc_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        y[c] = __uint_as_float(r0[c]);
        y[c + 32] = __uint_as_float(r1[c]);
      }
      if (p.bias) {
#pragma unroll
        for (int c = 0; c < kPoN; ++c) y[c] = __fadd_rn(y[c], __bfloat162float(p.bias[c]));
      }
#pragma unroll
      for (int c = 0; c < kPoN; ++c) y[c] = round_bf16(y[c]);     // proj_out's bf16 output
      if (row >= kPoTok) {
        uint4* dst = reinterpret_cast<uint4*>(negs + (row - kPoTok) * kPoN);
#pragma unroll
        for (int q = 0; q < kPoN / 8; ++q)
          dst[q] = make_uint4(pack_bf16x2(y[8 * q], y[8 * q + 1]), pack_bf16x2(y[8 * q + 2], y[8 * q + 3]),
                              pack_bf16x2(y[8 * q + 4], y[8 * q + 5]), pack_bf16x2(y[8 * q + 6], y[8 * q + 7]));
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");   // the four epilogue warps
    const int token = tok0 + row;
    if (got && row < kPoTok && token < p.rows) {
      const uint4* nrow = reinterpret_cast<const uint4*>(negs + row * kPoN);
      float ss_c = 0.0f, ss_m = 0.0f;
#pragma unroll
      for (int q = 0; q < kPoN / 8; ++q) {
        const uint4 nv = nrow[q];
        const uint32_t w[4] = {nv.x, nv.y, nv.z, nv.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float cv = y[8 * q + i];
          const float nn = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
          const float comb = round_bf16(__fadd_rn(nn, round_bf16(__fmul_rn(p.s, round_bf16(__fsub_rn(cv, nn))))));
          ss_c = __fmaf_rn(cv, cv, ss_c);
          ss_m = __fmaf_rn(comb, comb, ss_m);
          y[8 * q + i] = comb;
        }
      }
      const float ratio = round_bf16(__fdiv_rn(round_bf16(sqrtf(ss_c)), round_bf16(sqrtf(ss_m))));
      const float dt = __fsub_rn(p.sigmas[1], p.sigmas[0]);
      const uint4* lrow = reinterpret_cast<const uint4*>(p.lat + int64_t(token) * kPoN);
      uint4* orow = reinterpret_cast<uint4*>(p.out + int64_t(token) * kPoN);
#pragma unroll
      for (int q = 0; q < kPoN / 8; ++q) {
        const uint4 lv = lrow[q];
        const uint32_t w[4] = {lv.x, lv.y, lv.z, lv.w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float lat = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
          const float v = round_bf16(__fmul_rn(y[8 * q + i], ratio));
          o[i] = __fadd_rn(lat, round_bf16(__fmul_rn(dt, v)));
        }
        orow[q] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                             pack_bf16x2(o[6], o[7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kPoTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 po_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box {64, 64}, 128-byte swizzle.
int make_bf16_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols) {
  auto fn = po_encode_fn();
  if (!fn) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols * 2)};
  cuuint32_t box[2] = {uint32_t(kPoK), uint32_t(kPoTok)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return QIA_OK;
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_proj_out_cfg_euler(const void* y, const void* w, const void* bias, const void* latents, void* out,
                                      int64_t rows, int64_t k, int64_t n, float cfg_scale, const void* sigmas,
                                      void* stream) {
  if (!y || !w || !latents || !out || !sigmas)
    return set_error(QIA_ERR_INVALID, "qia_proj_out_cfg_euler: null pointer");
  if (rows <= 0 || k <= 0) return set_error(QIA_ERR_INVALID, "qia_proj_out_cfg_euler: rows=%lld k=%lld",
                                            (long long)rows, (long long)k);
  if (n != kPoN) return set_error(QIA_ERR_UNSUPPORTED, "qia_proj_out_cfg_euler: n=%lld (only 64)", (long long)n);
  if (k % kPoK || k > 65536) return set_error(QIA_ERR_UNSUPPORTED, "qia_proj_out_cfg_euler: k=%lld", (long long)k);
  if (rows > (int64_t(1) << 29)) return set_error(QIA_ERR_UNSUPPORTED, "qia_proj_out_cfg_euler: too many rows");
  if (!aligned(y, 16) || !aligned(w, 16) || !aligned(latents, 16) || !aligned(out, 16) || !aligned(sigmas, 4) ||
      (bias && !aligned(bias, 2)))
    return set_error(QIA_ERR_ALIGNMENT, "qia_proj_out_cfg_euler: misaligned pointer");
  static bool attr_done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(proj_out_cfg_euler_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kPoSmem);
      if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_done[dev] = true;
    }
  }
  CUtensorMap tm_y, tm_w;
  int rc = make_bf16_tmap(&tm_y, y, 2 * rows, k);
  if (rc) return rc;
  rc = make_bf16_tmap(&tm_w, w, n, k);
  if (rc) return rc;
  PoParams p;
  p.bias = (const __nv_bfloat16*)bias;
  p.lat = (const __nv_bfloat16*)latents;
  p.out = (__nv_bfloat16*)out;
  p.sigmas = (const float*)sigmas;
  p.rows = int(rows);
  p.k_blocks = int(k / kPoK);
  p.s = cfg_scale;
  const int64_t grid = (rows + kPoTok - 1) / kPoTok;
  proj_out_cfg_euler_kernel<<<unsigned(grid), 192, kPoSmem, as_stream(stream)>>>(tm_y, tm_w, p,
                                                                                 device_error_word());
  return check_launch("proj_out_cfg_euler_kernel");
}
