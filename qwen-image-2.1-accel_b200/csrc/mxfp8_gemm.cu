// Block-scaled MXFP8 GEMM on the 5th-generation tensor cores (tcgen05).
//
//   out[M, N] = epilogue( A[M, K] . B[N, K]^T ),  A, B: E4M3 codes with E8M0
//   scales per 1x32 block along K in the 128x4 blocked layout.
//
// Replaces torch._scaled_mm in MXFP8Linear.matmul (reference
// src/qwen_image_accel/optimizations/mxfp8.py:229-233) and adds the epilogues
// the dual-stream block needs (bias, GELU-tanh + MXFP8 requantization, gate +
// residual).
//
// Structure (one CTA per SM, persistent over output tiles, 6 warps):
//   warp 0      TMA producer: A tile 128x128 B, B tile BNx128 B (128-byte
//               swizzle) plus the 512-byte scale chunks (bulk copies) into a
//               STAGES-deep ring guarded by full/empty mbarriers.
//   warp 1      TMEM allocator and the single MMA-issuing thread: per K block
//               copies the scale chunks smem->TMEM (tcgen05.cp 32x128b.warpx4)
//               and issues four tcgen05.mma.kind::mxf8f6f4.block_scale (K=32
//               each, scale id = k step) into a TMEM accumulator; commits free
//               the smem stage and, per tile, publish the accumulator.
//   warps 2-9   epilogue: two warps per TMEM sub-partition (warp % 4), each
//               owning half of the tile's columns; tcgen05.ld 32 columns at a
//               time (one TMEM lane per output row), apply the epilogue in
//               registers, store to HBM. Eight warps keep the accurate-tanh
//               GELU epilogue shorter than the next tile's main loop.
// TMEM columns: NACC accumulators of BN columns (double-buffered when they
// fit, so the epilogue of tile i overlaps the MMAs of tile i+1), then the A
// scale slot (4 columns) and the B scale slot (4 per 128 rows of the tile).
// No TMA multicast and no clusters are used.
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace qia {
namespace {

enum Epi { kEpiBf16 = 0, kEpiGeluQuant = 1, kEpiGateResidual = 2, kEpiGeluBf16 = 3 };

struct EpiParams {
  __nv_bfloat16* out;          // [M, ldo] bf16 (kEpiBf16 / kEpiGeluBf16 / kEpiGateResidual)
  int64_t ldo;
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* gate;   // [M / rows_per_batch, N] (kEpiGateResidual)
  const __nv_bfloat16* resid;  // [M, ldo] (kEpiGateResidual; may alias out)
  int64_t rows_per_batch;
  uint8_t* q_values;           // [Mpad, N] e4m3 (kEpiGeluQuant)
  uint8_t* q_scales;           // blocked E8M0 (kEpiGeluQuant)
};

constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct Cfg {
  static constexpr int BM = 128, BK = 128;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int SFB_CHUNKS = (BN + 127) / 128;
  static constexpr int SF_BYTES = 512 + 512 * SFB_CHUNKS;
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES + SF_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGES = BN == 128 ? 6 : (BN == 192 ? 5 : 4);
  static constexpr int NACC = BN <= 192 ? 2 : 1;
  static constexpr int SFA_COL = NACC * BN;
  static constexpr int SFB_COL = SFA_COL + 4;
  static constexpr int TMEM_COLS = 512;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(SFB_COL + 4 * SFB_CHUNKS <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Instruction descriptor: E4M3 x E4M3 -> f32, E8M0 scales, K-major A and B,
// M = 128, N = BN; the scale ids (bits 4-5 and 29-30) are or-ed in per K step.
template <int BN>
__host__ __device__ constexpr uint32_t mxf8_idesc() {
  return (uint32_t(BN >> 3) << 17) | (1u << 23) | (uint32_t(128 >> 4) << 24);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
mxfp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                  const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, EpiParams ep, int M, int N,
                  int K, int* err) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bar_area = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + 127) / 128, n_tiles = N / BN, k_blocks = K / 128;
  const int num_tiles = m_tiles * n_tiles;
  const int kb_tiles = K / 128;  // 512-byte scale chunks per 128 rows

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), kEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int s = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / n_tiles, n_blk = tile % n_tiles;
        const int m0 = m_blk * 128, n0 = n_blk * BN;
        const uint8_t* sfa_tile = sfa + int64_t(m_blk) * kb_tiles * 512;
        const uint8_t* sfb_tile = sfb + int64_t(n0 >> 7) * kb_tiles * 512;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[s]), phase ^ 1, err)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_arrive_expect_tx(fb, C::A_BYTES + C::B_BYTES + C::SF_BYTES);
          tma_load_2d(smem_u32(st), &tmap_a, fb, kb * 128, m0);
          tma_load_2d(smem_u32(st + C::A_BYTES), &tmap_b, fb, kb * 128, n0);
          bulk_load(smem_u32(st + C::A_BYTES + C::B_BYTES), sfa_tile + kb * 512, 512, fb);
#pragma unroll
          for (int c = 0; c < C::SFB_CHUNKS; ++c)
            bulk_load(smem_u32(st + C::A_BYTES + C::B_BYTES + 512 + 512 * c),
                      sfb_tile + (int64_t(c) * kb_tiles + kb) * 512, 512, fb);
          ++issued;
          if (++s == C::STAGES) { s = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Let the copies already queued land before the CTA's shared memory goes away.
        for (int i = 0; i < C::STAGES && i < issued; ++i) {
          if (--s < 0) { s = C::STAGES - 1; phase ^= 1; }
          mbar_wait(smem_u32(&full[s]), phase, nullptr, 100000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int a = (C::NACC == 2) ? (it & 1) : 0;
        const uint32_t acc_phase = (C::NACC == 2) ? ((it >> 1) & 1) : (it & 1);
        if (!mbar_wait(smem_u32(&acc_empty[a]), acc_phase ^ 1, err)) { ok = false; break; }
        tc_fence_after();
        const int n0 = (tile % n_tiles) * BN;
        const uint32_t d_tmem = tmem_base + uint32_t(a * BN);
        const uint32_t sfa_tmem = tmem_base + C::SFA_COL;
        const uint32_t sfb_tmem = tmem_base + C::SFB_COL + uint32_t((n0 & 127) >> 5);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[s]), phase, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
          tc_cp_32x128b_warpx4(tmem_base + C::SFA_COL, smem_desc_sf(st + C::A_BYTES + C::B_BYTES));
#pragma unroll
          for (int c = 0; c < C::SFB_CHUNKS; ++c)
            tc_cp_32x128b_warpx4(tmem_base + C::SFB_COL + 4 * c,
                                 smem_desc_sf(st + C::A_BYTES + C::B_BYTES + 512 + 512 * c));
          const uint64_t adesc = smem_desc_k_sw128(st);
          const uint64_t bdesc = smem_desc_k_sw128(st + C::A_BYTES);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t idesc = mxf8_idesc<BN>() | (uint32_t(j) << 4) | (uint32_t(j) << 29);
            tc_mma_mxf8(d_tmem, adesc + uint64_t(2 * j), bdesc + uint64_t(2 * j), idesc, sfa_tmem, sfb_tmem,
                        (kb | j) != 0);
          }
          tc_commit(smem_u32(&empty[s]));
          if (++s == C::STAGES) { s = 0; phase ^= 1; }
        }
        if (ok) tc_commit(smem_u32(&acc_full[a]));
      }
      // drain: every MMA this thread issued has finished reading/writing TMEM
      tc_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, ok ? err : nullptr, 100000000ull);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;  // TMEM sub-partition this warp may access
    const int half = (warp - 2) / 4;  // which half of the tile's columns
    const int row_in_tile = sub * 32 + lane;
    constexpr int kChunks = BN / 64;  // 32-column chunks per warp
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int a = (C::NACC == 2) ? (it & 1) : 0;
      const uint32_t acc_phase = (C::NACC == 2) ? ((it >> 1) & 1) : (it & 1);
      // warp-uniform: the tcgen05.ld below needs all 32 lanes
      const bool got = __all_sync(0xffffffffu, mbar_wait(smem_u32(&acc_full[a]), acc_phase, err));
      if (!got) break;
      tc_fence_after();
      const int m0 = (tile / n_tiles) * 128, n0 = (tile % n_tiles) * BN;
      const int64_t row = m0 + row_in_tile;
      const bool live = row < M;
      const uint32_t t_row = tmem_base + (uint32_t(sub * 32) << 16) + uint32_t(a * BN);
#pragma unroll 1
      for (int jj = 0; jj < kChunks; ++jj) {
        const int j = half * kChunks + jj;
        uint32_t r[32];
        tc_ld_32x32b_x32(t_row + uint32_t(j * 32), r);
        tc_wait_ld();
        if (jj == kChunks - 1) {
          // all columns of this accumulator are in registers: hand it back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acc_empty[a]));
        }
        const int col = n0 + j * 32;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if (ep.bias) {
          const uint4* bp = reinterpret_cast<const uint4*>(ep.bias + col);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float bf[8];
            unpack8(__ldg(bp + q), bf);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[q * 8 + i] += bf[i];
          }
        }
        if (EPI == kEpiBf16 || EPI == kEpiGeluBf16) {
          if (live) {
            if (EPI == kEpiGeluBf16) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f32(round_bf16(v[i]));
            }
            uint4* op = reinterpret_cast<uint4*>(ep.out + row * ep.ldo + col);
#pragma unroll
            for (int q = 0; q < 4; ++q) op[q] = pack8(&v[q * 8]);
          }
        } else if (EPI == kEpiGateResidual) {
          if (live) {
            const int64_t b = row / ep.rows_per_batch;
            const uint4* gp = reinterpret_cast<const uint4*>(ep.gate + b * N + col);
            const uint4* hp = reinterpret_cast<const uint4*>(ep.resid + row * ep.ldo + col);
            uint4* op = reinterpret_cast<uint4*>(ep.out + row * ep.ldo + col);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float g[8], h[8], o[8];
              unpack8(__ldg(gp + q), g);
              unpack8(hp[q], h);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                o[i] = __fadd_rn(h[i], round_bf16(__fmul_rn(g[i], round_bf16(v[q * 8 + i]))));
              op[q] = pack8(o);
            }
          }
        } else {  // kEpiGeluQuant: the 32 columns are exactly one MX block of the next GEMM's K
          float amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = live ? round_bf16(gelu_tanh_f32(round_bf16(v[i]))) : 0.0f;
            amax = fmaxf(amax, fabsf(v[i]));
          }
          const int e = mx_exponent(amax);
          const float inv = mx_inverse_scale(e);
          uint4 c0, c1;
          c0.x = cvt_e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
          c0.y = cvt_e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
          c0.z = cvt_e4m3x4(v[8] * inv, v[9] * inv, v[10] * inv, v[11] * inv);
          c0.w = cvt_e4m3x4(v[12] * inv, v[13] * inv, v[14] * inv, v[15] * inv);
          c1.x = cvt_e4m3x4(v[16] * inv, v[17] * inv, v[18] * inv, v[19] * inv);
          c1.y = cvt_e4m3x4(v[20] * inv, v[21] * inv, v[22] * inv, v[23] * inv);
          c1.z = cvt_e4m3x4(v[24] * inv, v[25] * inv, v[26] * inv, v[27] * inv);
          c1.w = cvt_e4m3x4(v[28] * inv, v[29] * inv, v[30] * inv, v[31] * inv);
          uint4* qp = reinterpret_cast<uint4*>(ep.q_values + row * int64_t(N) + col);
          qp[0] = c0;
          qp[1] = c1;
          ep.q_scales[mx_scale_offset(row, col >> 5, N >> 7)] = uint8_t(e);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D uint8 tensor map over a row-major [rows, cols] matrix, box {128, box_rows},
// 128-byte swizzle.
int make_tmap(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols)};
  cuuint32_t box[2] = {128u, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return QIA_OK;
}

template <int BN, int EPI>
int launch_gemm(const void* a, const void* sa, const void* b, const void* sb, const EpiParams& ep, int64_t M,
                int64_t N, int64_t K, cudaStream_t st) {
  using C = Cfg<BN>;
  static bool attr_done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(mxfp8_gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::SMEM);
      if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_done[dev] = true;
    }
  }
  const int64_t m_pad = (M + 127) / 128 * 128;
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, a, m_pad, K, 128);
  if (rc) return rc;
  rc = make_tmap(&tb, b, N, K, BN);
  if (rc) return rc;
  const int64_t tiles = (m_pad / 128) * (N / BN);
  int64_t grid = sm_count();
  if (grid > tiles) grid = tiles;
  mxfp8_gemm_kernel<BN, EPI><<<unsigned(grid), kGemmThreads, C::SMEM, st>>>(
      ta, tb, (const uint8_t*)sa, (const uint8_t*)sb, ep, int(M), int(N), int(K), device_error_word());
  return check_launch("mxfp8_gemm_kernel");
}

int pick_bn(int64_t M, int64_t N) {
  // QIA_GEMM_BN (128, 192 or 256) pins the tile width, for tuning and tests.
  const char* env = getenv("QIA_GEMM_BN");
  const int forced = env ? atoi(env) : 0;
  if ((forced == 128 || forced == 192 || forced == 256) && N % forced == 0) return forced;
  // Prefer the tile width with the best last-wave occupancy over the SMs.
  const int64_t m_tiles = (M + 127) / 128;
  const int sms = sm_count();
  int best = 0;
  double best_eff = -1.0;
  for (int bn : {192, 256, 128}) {
    if (N % bn) continue;
    const int64_t tiles = m_tiles * (N / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    // double-buffered accumulators hide the epilogue; single-buffered do not
    const double eff = double(tiles) / double(waves * sms) * (bn == 256 ? 0.92 : 1.0) * (bn == 128 ? 0.95 : 1.0);
    if (eff > best_eff + 1e-9) { best_eff = eff; best = bn; }
  }
  return best;
}

template <int EPI>
int dispatch(const void* a, const void* sa, const void* b, const void* sb, const EpiParams& ep, int64_t M, int64_t N,
             int64_t K, void* stream, const char* who) {
  if (!a || !sa || !b || !sb) return set_error(QIA_ERR_INVALID, "%s: null operand", who);
  if (M <= 0 || N <= 0 || K <= 0) return set_error(QIA_ERR_INVALID, "%s: M=%lld N=%lld K=%lld", who, (long long)M,
                                                   (long long)N, (long long)K);
  if (K % 128 || N % 128) return set_error(QIA_ERR_UNSUPPORTED, "%s: K and N must be multiples of 128", who);
  if (M > (1LL << 30) || K > (1LL << 20) || N > (1LL << 20)) return set_error(QIA_ERR_UNSUPPORTED, "%s: too large", who);
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sa, 16) || !aligned(sb, 16))
    return set_error(QIA_ERR_ALIGNMENT, "%s: operands must be 16-byte aligned", who);
  const int bn = pick_bn(M, N);
  cudaStream_t st = as_stream(stream);
  switch (bn) {
    case 128: return launch_gemm<128, EPI>(a, sa, b, sb, ep, M, N, K, st);
    case 192: return launch_gemm<192, EPI>(a, sa, b, sb, ep, M, N, K, st);
    case 256: return launch_gemm<256, EPI>(a, sa, b, sb, ep, M, N, K, st);
    default: return set_error(QIA_ERR_UNSUPPORTED, "%s: N=%lld has no supported tile width", who, (long long)N);
  }
}

int check_out(const void* out, int64_t ldo, int64_t N, const char* who) {
  if (!out) return set_error(QIA_ERR_INVALID, "%s: null output", who);
  if (ldo < N || ldo % 8) return set_error(QIA_ERR_INVALID, "%s: ldo must be >= N and a multiple of 8", who);
  if (!aligned(out, 16)) return set_error(QIA_ERR_ALIGNMENT, "%s: output must be 16-byte aligned", who);
  return QIA_OK;
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_mxfp8_gemm(const void* a_values, const void* a_scales, const void* b_values, const void* b_scales,
                              const void* bias, void* out, int64_t m, int64_t n, int64_t k, int64_t ldo,
                              void* stream) {
  int rc = check_out(out, ldo, n, "qia_mxfp8_gemm");
  if (rc) return rc;
  if (bias && !aligned(bias, 16)) return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_gemm: bias alignment");
  EpiParams ep{};
  ep.out = (__nv_bfloat16*)out;
  ep.ldo = ldo;
  ep.bias = (const __nv_bfloat16*)bias;
  return dispatch<kEpiBf16>(a_values, a_scales, b_values, b_scales, ep, m, n, k, stream, "qia_mxfp8_gemm");
}

extern "C" int qia_mxfp8_gemm_gelu(const void* a_values, const void* a_scales, const void* b_values,
                                   const void* b_scales, const void* bias, void* out, int64_t m, int64_t n, int64_t k,
                                   int64_t ldo, void* stream) {
  int rc = check_out(out, ldo, n, "qia_mxfp8_gemm_gelu");
  if (rc) return rc;
  if (bias && !aligned(bias, 16)) return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_gemm_gelu: bias alignment");
  EpiParams ep{};
  ep.out = (__nv_bfloat16*)out;
  ep.ldo = ldo;
  ep.bias = (const __nv_bfloat16*)bias;
  return dispatch<kEpiGeluBf16>(a_values, a_scales, b_values, b_scales, ep, m, n, k, stream, "qia_mxfp8_gemm_gelu");
}

extern "C" int qia_mxfp8_gemm_gelu_quant(const void* a_values, const void* a_scales, const void* b_values,
                                         const void* b_scales, const void* bias, void* q_values, void* q_scales,
                                         int64_t m, int64_t n, int64_t k, void* stream) {
  if (!q_values || !q_scales) return set_error(QIA_ERR_INVALID, "qia_mxfp8_gemm_gelu_quant: null output");
  if (!aligned(q_values, 16) || (bias && !aligned(bias, 16)))
    return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_gemm_gelu_quant: alignment");
  EpiParams ep{};
  ep.bias = (const __nv_bfloat16*)bias;
  ep.q_values = (uint8_t*)q_values;
  ep.q_scales = (uint8_t*)q_scales;
  return dispatch<kEpiGeluQuant>(a_values, a_scales, b_values, b_scales, ep, m, n, k, stream,
                                 "qia_mxfp8_gemm_gelu_quant");
}

extern "C" int qia_mxfp8_gemm_gate_residual(const void* a_values, const void* a_scales, const void* b_values,
                                            const void* b_scales, const void* bias, const void* gate,
                                            const void* resid, void* out, int64_t m, int64_t n, int64_t k,
                                            int64_t ldo, int64_t rows_per_batch, void* stream) {
  int rc = check_out(out, ldo, n, "qia_mxfp8_gemm_gate_residual");
  if (rc) return rc;
  if (!gate || !resid || rows_per_batch <= 0)
    return set_error(QIA_ERR_INVALID, "qia_mxfp8_gemm_gate_residual: gate/resid/rows_per_batch");
  if (!aligned(gate, 16) || !aligned(resid, 16) || (bias && !aligned(bias, 16)))
    return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_gemm_gate_residual: alignment");
  EpiParams ep{};
  ep.out = (__nv_bfloat16*)out;
  ep.ldo = ldo;
  ep.bias = (const __nv_bfloat16*)bias;
  ep.gate = (const __nv_bfloat16*)gate;
  ep.resid = (const __nv_bfloat16*)resid;
  ep.rows_per_batch = rows_per_batch;
  return dispatch<kEpiGateResidual>(a_values, a_scales, b_values, b_scales, ep, m, n, k, stream,
                                    "qia_mxfp8_gemm_gate_residual");
}
