// Block-scaled MXFP8 GEMM on the 5th-generation tensor cores (tcgen05).
//
//   out[M, N] = epilogue( A[M, K] . B[N, K]^T ),  A, B: E4M3 codes with E8M0
//   scales per 1x32 block along K in the 128x4 blocked layout.
//
// Replaces torch._scaled_mm in MXFP8Linear.matmul (reference
// src/qwen_image_accel/optimizations/mxfp8.py:32-36) and adds the epilogues
// the dual-stream block needs (bias, GELU-tanh + MXFP8 requantization, gate +
// residual).
//
// Structure (one CTA per SM, persistent over output tiles, 10 warps):
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
//               registers, store to HBM. The GELU epilogues use the
//               two-MUFU sigmoid form of GELU-tanh (gelu_tanh_fast) and run on
//               BN=192 tiles, whose double-buffered accumulators let the
//               epilogue of one tile overlap the main loop of the next.
//
// TMEM columns: NACC accumulators of BN columns (double-buffered when they
// fit, so the epilogue of tile i overlaps the MMAs of tile i+1; with the one
// accumulator of BN=256 the epilogue warps take all their columns into
// registers and release it before the epilogue math), then
// SF_SLOTS scale slots used round-robin per K block, each the A scales (4
// columns) and the B scales (4 per 128 rows of the tile).
// No TMA multicast is used anywhere.
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace qia {
namespace {

enum Epi { kEpiBf16 = 0, kEpiGeluQuant = 1, kEpiGateResidual = 2, kEpiGeluBf16 = 3, kEpiSwigluQuant = 4 };

struct EpiParams {
  __nv_bfloat16* out;          // [M, ldo] bf16 (kEpiBf16 / kEpiGeluBf16 / kEpiGateResidual)
  int64_t ldo;
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* gate;   // [M / rows_per_batch, N] (kEpiGateResidual)
  const __nv_bfloat16* resid;  // [M, ldo] (kEpiGateResidual; may alias out)
  int64_t rows_per_batch;
  uint8_t* q_values;           // [Mpad, N] e4m3 (kEpiGeluQuant); [Mpad, N/2] (kEpiSwigluQuant)
  uint8_t* q_scales;           // blocked E8M0 (kEpiGeluQuant, kEpiSwigluQuant)
  int wide;                    // out/resid/q_values rows allow 32-byte accesses
};

// One or two GEMMs with the same N, K, tile width and epilogue kind run as
// one persistent launch (the dual-stream block's image and text projections):
// output tiles [0, tiles0) belong to problem 0, [tiles0, num_tiles) to
// problem 1, so the small text GEMM fills the image GEMM's last wave instead
// of running as a separate, mostly idle launch.
struct GemmGroup {
  const uint8_t* sfa0;
  const uint8_t* sfb0;
  const uint8_t* sfa1;
  const uint8_t* sfb1;
  EpiParams ep0, ep1;
  int M0, M1;
  int tiles0, num_tiles;
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
  // scale-factor slots in TMEM, used round-robin per K block so that the copy
  // for block kb+1 never overwrites scales the MMAs of block kb still read
  static constexpr int SF_SLOTS = 4;
  static constexpr int SF_COLS = 16;       // A scales at +0, B scales at +8 (8-column aligned)
  static constexpr int SFB_OFF = 8;
  static constexpr int SFA_COL = NACC * BN;   // slot s: A at SFA_COL + s*SF_COLS, B SFB_OFF columns later
  static constexpr int TMEM_COLS = 512;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(SFA_COL + SF_SLOTS * SF_COLS <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Instruction descriptor: E4M3 x E4M3 -> f32, E8M0 scales, K-major A and B,
// M = 128, N = BN; the scale ids (bits 4-5 and 29-30) are or-ed in per K step.
template <int BN>
__host__ __device__ constexpr uint32_t mxf8_idesc() {
  return (uint32_t(BN >> 3) << 17) | (1u << 23) | (uint32_t(128 >> 4) << 24);
}

// Epilogue of one 32-column chunk of an accumulator row (v: fp32 sums).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(float (&v)[32], const EpiParams& ep, int64_t row, int col, bool live,
                                               int N) {
  if (ep.bias) {
    const uint4* bp = reinterpret_cast<const uint4*>(ep.bias + col);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float bf[8];
      unpack8(__ldg(bp + q), bf);
#pragma unroll
      for (int i = 0; i < 8; i += 2)
        f2_unpack(f2_add(f2_pack(v[q * 8 + i], v[q * 8 + i + 1]), f2_pack(bf[i], bf[i + 1])), v[q * 8 + i],
                  v[q * 8 + i + 1]);
    }
  }
  // Each thread owns one row: a 32-column chunk is 64 contiguous bytes of bf16,
  // written (and, for the residual, read) as two full 32-byte sectors when the
  // row start allows it, else as four 16-byte pieces.
  if (EPI == kEpiBf16 || EPI == kEpiGeluBf16) {
    if (live) {
      if (EPI == kEpiGeluBf16) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          round_bf16_x2(v[i], v[i + 1]);
          gelu_tanh_fast_x2(v[i], v[i + 1]);
        }
      }
      uint4 pk[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) pk[q] = pack8(&v[q * 8]);
      uint4* op = reinterpret_cast<uint4*>(ep.out + row * ep.ldo + col);
      if (ep.wide) {
        st_global_v8(op, pk[0], pk[1]);
        st_global_v8(op + 2, pk[2], pk[3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) op[q] = pk[q];
      }
    }
  } else if (EPI == kEpiGateResidual) {
    if (live) {
      const int64_t b = row / ep.rows_per_batch;
      const uint4* gp = reinterpret_cast<const uint4*>(ep.gate + b * N + col);
      const uint4* hp = reinterpret_cast<const uint4*>(ep.resid + row * ep.ldo + col);
      uint4* op = reinterpret_cast<uint4*>(ep.out + row * ep.ldo + col);
      uint4 hv[4], ov[4];
      if (ep.wide) {
        ld_global_v8(hp, hv[0], hv[1]);
        ld_global_v8(hp + 2, hv[2], hv[3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) hv[q] = hp[q];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float g[8], h[8], o[8];
        unpack8(__ldg(gp + q), g);
        unpack8(hv[q], h);
        // o = h + bf16(g * bf16(v)), on lane pairs
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float y0 = v[q * 8 + i], y1 = v[q * 8 + i + 1];
          round_bf16_x2(y0, y1);
          f2_unpack(f2_mul(f2_pack(g[i], g[i + 1]), f2_pack(y0, y1)), y0, y1);
          round_bf16_x2(y0, y1);
          f2_unpack(f2_add(f2_pack(h[i], h[i + 1]), f2_pack(y0, y1)), o[i], o[i + 1]);
        }
        ov[q] = pack8(o);
      }
      if (ep.wide) {
        st_global_v8(op, ov[0], ov[1]);
        st_global_v8(op + 2, ov[2], ov[3]);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) op[q] = ov[q];
      }
    }
  } else if (EPI == kEpiSwigluQuant) {
    // handled per chunk pair (epilogue_swiglu_pair)
  } else {  // kEpiGeluQuant: the 32 columns are exactly one MX block of the next GEMM's K
    // bf16 round -> GELU -> bf16 round -> |max|, on lane pairs (f32x2)
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float x0 = v[i], x1 = v[i + 1];
      round_bf16_x2(x0, x1);
      gelu_tanh_fast_x2(x0, x1);
      round_bf16_x2(x0, x1);
      v[i] = live ? x0 : 0.0f;
      v[i + 1] = live ? x1 : 0.0f;
      amax = fmaxf(fmaxf(amax, fabsf(v[i])), fabsf(v[i + 1]));
    }
    const int e = mx_exponent(amax);
    const float inv = mx_inverse_scale(e);
    const uint64_t inv2 = f2_pack(inv, inv);
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float y0, y1, y2, y3;
      f2_unpack(f2_mul(f2_pack(v[4 * q], v[4 * q + 1]), inv2), y0, y1);
      f2_unpack(f2_mul(f2_pack(v[4 * q + 2], v[4 * q + 3]), inv2), y2, y3);
      w[q] = cvt_e4m3x4(y0, y1, y2, y3);
    }
    uint4 c0 = make_uint4(w[0], w[1], w[2], w[3]), c1 = make_uint4(w[4], w[5], w[6], w[7]);
    uint4* qp = reinterpret_cast<uint4*>(ep.q_values + row * int64_t(N) + col);
    if (ep.wide) {
      st_global_v8(qp, c0, c1);
    } else {
      qp[0] = c0;
      qp[1] = c1;
    }
    ep.q_scales[mx_scale_offset(row, col >> 5, N >> 7)] = uint8_t(e);
  }
}

// SwiGLU epilogue of one chunk pair: the B operand stacks the gate and value
// projections interleaved every 32 rows, so output columns [64 j, 64 j + 32)
// are gate columns [32 j, 32 j + 32) and the next 32 the matching value
// columns. Both are rounded to bf16 (the GEMMs' bf16 outputs), combined as
// bf16(silu(g) * v) and quantized as one MX block of column block j of the
// [Mpad, N/2] activation -- the arithmetic of a bf16 GEMM pair followed by
// the SwiGLU + MXFP8 quantizer.
__device__ __forceinline__ void epilogue_swiglu_pair(const float (&vg)[32], const float (&vv)[32],
                                                     const EpiParams& ep, int64_t row, int out_col, bool live,
                                                     int n_out) {
  float y[32];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float g = round_bf16(vg[i]), v = round_bf16(vv[i]);
    y[i] = live ? round_bf16(__fmul_rn(silu_ref(g), v)) : 0.0f;
    amax = fmaxf(amax, fabsf(y[i]));
  }
  const int e = mx_exponent(amax);
  const float inv = mx_inverse_scale(e);
  const uint64_t inv2 = f2_pack(inv, inv);
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float y0, y1, y2, y3;
    f2_unpack(f2_mul(f2_pack(y[4 * q], y[4 * q + 1]), inv2), y0, y1);
    f2_unpack(f2_mul(f2_pack(y[4 * q + 2], y[4 * q + 3]), inv2), y2, y3);
    w[q] = cvt_e4m3x4(y0, y1, y2, y3);
  }
  uint4 c0 = make_uint4(w[0], w[1], w[2], w[3]), c1 = make_uint4(w[4], w[5], w[6], w[7]);
  uint4* qp = reinterpret_cast<uint4*>(ep.q_values + row * int64_t(n_out) + out_col);
  if (ep.wide) {
    st_global_v8(qp, c0, c1);
  } else {
    qp[0] = c0;
    qp[1] = c1;
  }
  ep.q_scales[mx_scale_offset(row, out_col >> 5, n_out >> 7)] = uint8_t(e);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
mxfp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a0, const __grid_constant__ CUtensorMap tmap_b0,
                  const __grid_constant__ CUtensorMap tmap_a1, const __grid_constant__ CUtensorMap tmap_b1,
                  const GemmGroup g, int N, int K, int* err) {
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
  const int n_tiles = N / BN, k_blocks = K / 128;
  const int num_tiles = g.num_tiles;
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
    prefetch_tmap(&tmap_a0);
    prefetch_tmap(&tmap_b0);
    if (g.num_tiles > g.tiles0) {
      prefetch_tmap(&tmap_a1);
      prefetch_tmap(&tmap_b1);
    }
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
        const bool second = tile >= g.tiles0;
        const int lt = second ? tile - g.tiles0 : tile;
        const int m_blk = lt / n_tiles, n_blk = lt % n_tiles;
        const int m0 = m_blk * 128, n0 = n_blk * BN;
        const CUtensorMap* tmap_a = second ? &tmap_a1 : &tmap_a0;
        const CUtensorMap* tmap_b = second ? &tmap_b1 : &tmap_b0;
        const uint8_t* sfa_tile = (second ? g.sfa1 : g.sfa0) + int64_t(m_blk) * kb_tiles * 512;
        const uint8_t* sfb_tile = (second ? g.sfb1 : g.sfb0) + int64_t(n0 >> 7) * kb_tiles * 512;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[s]), phase ^ 1, err)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          const uint32_t fb = smem_u32(&full[s]);
          mbar_arrive_expect_tx(fb, C::A_BYTES + C::B_BYTES + C::SF_BYTES);
          tma_load_2d(smem_u32(st), tmap_a, fb, kb * 128, m0);
          tma_load_2d(smem_u32(st + C::A_BYTES), tmap_b, fb, kb * 128, n0);
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
    // Kept to a few instructions per K block (this warp shares its SM
    // sub-partition with busy epilogue warps): the stage's descriptors advance
    // by a constant (STAGE_BYTES/16 in the start-address field), the scale
    // slot and barrier addresses by fixed strides.
    if (lane == 0) {
      constexpr uint32_t kStageDesc = C::STAGE_BYTES >> 4;
      const uint32_t smem0 = smem_u32(smem);
      const uint64_t adesc0 = smem_desc_k_sw128(smem0);
      const uint64_t bdesc0 = smem_desc_k_sw128(smem0 + C::A_BYTES);
      const uint64_t sfdesc0 = smem_desc_sf(smem0 + C::A_BYTES + C::B_BYTES);
      const uint32_t full0 = smem_u32(&full[0]), empty0 = smem_u32(&empty[0]);
      const uint32_t sf0 = tmem_base + uint32_t(C::SFA_COL);
      int s = 0, sf_slot = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int a = (C::NACC == 2) ? (it & 1) : 0;
        const uint32_t acc_phase = (C::NACC == 2) ? ((it >> 1) & 1) : (it & 1);
        if (!mbar_wait(smem_u32(&acc_empty[a]), acc_phase ^ 1, err)) { ok = false; break; }
        tc_fence_after();
        const int n0 = ((tile >= g.tiles0 ? tile - g.tiles0 : tile) % n_tiles) * BN;
        const uint32_t d_tmem = tmem_base + uint32_t(a * BN);
        // BN=192 tiles at odd multiples of 64 start 2 columns into the chunk
        const uint32_t sfb_shift = uint32_t(C::SFB_OFF + ((n0 & 127) >> 5));
        for (int kb = 0; kb < k_blocks; ++kb) {
          // TMA completion on `full` orders the stage's bytes for the MMAs
          // (async proxy on both sides): no tcgen05 fence per K block
          if (!mbar_wait(full0 + 8u * uint32_t(s), phase, err)) { ok = false; break; }
          const uint64_t off = uint64_t(uint32_t(s) * kStageDesc);
          const uint32_t sfa_tmem = sf0 + uint32_t(sf_slot * C::SF_COLS);
          if (++sf_slot == C::SF_SLOTS) sf_slot = 0;
          tc_cp_32x128b_warpx4(sfa_tmem, sfdesc0 + off);
#pragma unroll
          for (int c = 0; c < C::SFB_CHUNKS; ++c)
            tc_cp_32x128b_warpx4(sfa_tmem + uint32_t(C::SFB_OFF + 4 * c), sfdesc0 + off + uint64_t(32 + 32 * c));
          const uint64_t adesc = adesc0 + off, bdesc = bdesc0 + off;
          const uint32_t sfb_tmem = sfa_tmem + sfb_shift;
          tc_mma_mxf8(d_tmem, adesc, bdesc, mxf8_idesc<BN>(), sfa_tmem, sfb_tmem, kb != 0);
#pragma unroll
          for (int j = 1; j < 4; ++j)
            tc_mma_mxf8(d_tmem, adesc + uint64_t(2 * j), bdesc + uint64_t(2 * j),
                        mxf8_idesc<BN>() | (uint32_t(j) << 4) | (uint32_t(j) << 29), sfa_tmem, sfb_tmem, 1u);
          tc_commit(empty0 + 8u * uint32_t(s));
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
    static_assert(EPI != kEpiSwigluQuant || kChunks % 2 == 0, "SwiGLU pairs need an even chunk count");
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int a = (C::NACC == 2) ? (it & 1) : 0;
      const uint32_t acc_phase = (C::NACC == 2) ? ((it >> 1) & 1) : (it & 1);
      // warp-uniform: the tcgen05.ld below needs all 32 lanes
      const bool got = __all_sync(0xffffffffu, mbar_wait(smem_u32(&acc_full[a]), acc_phase, err));
      if (!got) break;
      tc_fence_after();
      const bool second = tile >= g.tiles0;
      const int lt = second ? tile - g.tiles0 : tile;
      const int m0 = (lt / n_tiles) * 128, n0 = (lt % n_tiles) * BN;
      const EpiParams& ep = second ? g.ep1 : g.ep0;
      const int64_t row = m0 + row_in_tile;
      const bool live = row < (second ? g.M1 : g.M0);
      const uint32_t t_row = tmem_base + (uint32_t(sub * 32) << 16) + uint32_t(a * BN);
      if constexpr (C::NACC == 1) {
        // one accumulator: the next tile's MMAs wait for it, so take all of
        // this warp's columns into registers and hand it back before the math
        uint32_t r[kChunks][32];
#pragma unroll
        for (int jj = 0; jj < kChunks; ++jj) tc_ld_32x32b_x32(t_row + uint32_t((half * kChunks + jj) * 32), r[jj]);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acc_empty[a]));
        if constexpr (EPI == kEpiSwigluQuant) {
#pragma unroll
          for (int jj = 0; jj < kChunks; jj += 2) {
            float vg[32], vv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              vg[i] = __uint_as_float(r[jj][i]);
              vv[i] = __uint_as_float(r[jj + 1][i]);
            }
            epilogue_swiglu_pair(vg, vv, ep, row, (n0 + (half * kChunks + jj) * 32) / 2, live, N / 2);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < kChunks; ++jj) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[jj][i]);
            epilogue_chunk<EPI>(v, ep, row, n0 + (half * kChunks + jj) * 32, live, N);
          }
        }
      } else if constexpr (EPI == kEpiSwigluQuant) {
#pragma unroll 1
        for (int jj = 0; jj < kChunks; jj += 2) {
          const int j = half * kChunks + jj;
          uint32_t rg[32], rv[32];
          tc_ld_32x32b_x32(t_row + uint32_t(j * 32), rg);
          tc_ld_32x32b_x32(t_row + uint32_t((j + 1) * 32), rv);
          tc_wait_ld();
          if (jj == kChunks - 2) {
            // all columns of this accumulator are in registers: hand it back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty[a]));
          }
          float vg[32], vv[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            vg[i] = __uint_as_float(rg[i]);
            vv[i] = __uint_as_float(rv[i]);
          }
          epilogue_swiglu_pair(vg, vv, ep, row, (n0 + j * 32) / 2, live, N / 2);
        }
      } else {
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
          epilogue_chunk<EPI>(v, ep, row, col, live, N);
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

// One GEMM of a group as the host sees it.
struct Problem {
  const void* a;
  const void* sa;
  const void* b;
  const void* sb;
  EpiParams ep;
  int64_t M;
};

template <int BN, int EPI>
int launch_gemm(const Problem* pr, int count, int64_t N, int64_t K, cudaStream_t st) {
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
  CUtensorMap ta[2], tb[2];
  int64_t tiles[2] = {0, 0};
  for (int i = 0; i < count; ++i) {
    const int64_t m_pad = (pr[i].M + 127) / 128 * 128;
    int rc = make_tmap(&ta[i], pr[i].a, m_pad, K, 128);
    if (rc) return rc;
    rc = make_tmap(&tb[i], pr[i].b, N, K, BN);
    if (rc) return rc;
    tiles[i] = (m_pad / 128) * (N / BN);
  }
  if (count == 1) {
    ta[1] = ta[0];
    tb[1] = tb[0];
  }
  GemmGroup g;
  g.sfa0 = (const uint8_t*)pr[0].sa;
  g.sfb0 = (const uint8_t*)pr[0].sb;
  g.ep0 = pr[0].ep;
  g.M0 = int(pr[0].M);
  const Problem& p1 = pr[count - 1];
  g.sfa1 = (const uint8_t*)p1.sa;
  g.sfb1 = (const uint8_t*)p1.sb;
  g.ep1 = p1.ep;
  g.M1 = int(p1.M);
  g.tiles0 = int(tiles[0]);
  g.num_tiles = int(tiles[0] + tiles[1]);
  int64_t grid = sm_count();
  if (grid > g.num_tiles) grid = g.num_tiles;
  mxfp8_gemm_kernel<BN, EPI><<<unsigned(grid), kGemmThreads, C::SMEM, st>>>(ta[0], tb[0], ta[1], tb[1], g, int(N),
                                                                            int(K), device_error_word());
  return check_launch("mxfp8_gemm_kernel");
}

// 2-D uint8 view [rows, 256] of a scale-factor array (512-byte chunks = two
// rows), box {256, 2}, no swizzle: one TMA copy per chunk.
int make_sf_tmap(CUtensorMap* map, const void* base, int64_t bytes) {
  auto fn = encode_fn();
  if (!fn) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {256u, cuuint64_t(bytes / 256)};
  cuuint64_t strides[1] = {256u};
  cuuint32_t box[2] = {256u, 2u};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QIA_ERR_CUDA, "cuTensorMapEncodeTiled (scales) failed (%d)", int(r));
  return QIA_OK;
}

int pick_bn(int64_t M, int64_t N, bool heavy_epilogue, bool even_chunks = false) {
  // QIA_GEMM_BN (128, 192 or 256) pins the tile width, for tuning and tests.
  const char* env = getenv("QIA_GEMM_BN");
  const int forced = env ? atoi(env) : 0;
  if ((forced == 128 || (forced == 192 && !even_chunks) || forced == 256) && N % forced == 0) return forced;
  (void)heavy_epilogue;   // the f32x2 GELU epilogues keep up with BN=256 main loops
  // Prefer the tile width with the best last-wave occupancy over the SMs.
  const int64_t m_tiles = (M + 127) / 128;
  const int sms = sm_count();
  int best = 0;
  double best_eff = -1.0;
  for (int bn : {192, 256, 128}) {
    if (N % bn || (even_chunks && bn == 192)) continue;   // the SwiGLU epilogue pairs 32-column chunks
    const int64_t tiles = m_tiles * (N / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    // measured per-tile efficiency on B200: BN=256 (one accumulator, released
    // before the epilogue math) > 192 > 128
    const double eff = double(tiles) / double(waves * sms) * (bn == 192 ? 0.8 : 1.0) * (bn == 128 ? 0.7 : 1.0);
    if (eff > best_eff + 1e-9) { best_eff = eff; best = bn; }
  }
  return best;
}

template <int EPI>
int dispatch(const Problem* in, int count, int64_t N, int64_t K, void* stream, const char* who) {
  if (count < 1 || count > 2) return set_error(QIA_ERR_INVALID, "%s: 1 or 2 problems per launch", who);
  if (N <= 0 || K <= 0) return set_error(QIA_ERR_INVALID, "%s: N=%lld K=%lld", who, (long long)N, (long long)K);
  if (K % 128 || N % 128) return set_error(QIA_ERR_UNSUPPORTED, "%s: K and N must be multiples of 128", who);
  if (K > (1LL << 20) || N > (1LL << 20)) return set_error(QIA_ERR_UNSUPPORTED, "%s: too large", who);
  Problem pr[2];
  int64_t m_tiles = 0;
  for (int i = 0; i < count; ++i) {
    const Problem& p = in[i];
    if (!p.a || !p.sa || !p.b || !p.sb) return set_error(QIA_ERR_INVALID, "%s: null operand", who);
    if (p.M <= 0 || p.M > (1LL << 30)) return set_error(QIA_ERR_INVALID, "%s: M=%lld", who, (long long)p.M);
    if (!aligned(p.a, 16) || !aligned(p.b, 16) || !aligned(p.sa, 16) || !aligned(p.sb, 16))
      return set_error(QIA_ERR_ALIGNMENT, "%s: operands must be 16-byte aligned", who);
    pr[i] = p;
    const EpiParams& ep = p.ep;
    pr[i].ep.wide = (!ep.out || (aligned(ep.out, 32) && ep.ldo % 16 == 0)) && (!ep.resid || aligned(ep.resid, 32)) &&
                    (!ep.q_values || aligned(ep.q_values, 32));
    m_tiles += (p.M + 127) / 128;
  }
  if (m_tiles * 128 > (1LL << 30)) return set_error(QIA_ERR_UNSUPPORTED, "%s: too large", who);
  cudaStream_t st = as_stream(stream);
  // the tile width is chosen for the group's total M tiles
  const int bn = pick_bn(m_tiles * 128, N, EPI == kEpiGeluQuant || EPI == kEpiGeluBf16, EPI == kEpiSwigluQuant);
  switch (bn) {
    case 128: return launch_gemm<128, EPI>(pr, count, N, K, st);
    case 192:
      if constexpr (EPI != kEpiSwigluQuant) return launch_gemm<192, EPI>(pr, count, N, K, st);
      break;
    case 256: return launch_gemm<256, EPI>(pr, count, N, K, st);
    default: break;
  }
  return set_error(QIA_ERR_UNSUPPORTED, "%s: N=%lld has no supported tile width", who, (long long)N);
}

template <int EPI>
int dispatch(const void* a, const void* sa, const void* b, const void* sb, const EpiParams& ep, int64_t M, int64_t N,
             int64_t K, void* stream, const char* who) {
  Problem p{a, sa, b, sb, ep, M};
  return dispatch<EPI>(&p, 1, N, K, stream, who);
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

extern "C" int qia_mxfp8_gemm_swiglu_quant(const void* a_values, const void* a_scales, const void* b_values,
                                           const void* b_scales, void* q_values, void* q_scales, int64_t m,
                                           int64_t n, int64_t k, void* stream) {
  if (!q_values || !q_scales) return set_error(QIA_ERR_INVALID, "qia_mxfp8_gemm_swiglu_quant: null output");
  if (n % 256) return set_error(QIA_ERR_UNSUPPORTED, "qia_mxfp8_gemm_swiglu_quant: n must be a multiple of 256");
  if (!aligned(q_values, 16)) return set_error(QIA_ERR_ALIGNMENT, "qia_mxfp8_gemm_swiglu_quant: q_values alignment");
  EpiParams ep{};
  ep.q_values = (uint8_t*)q_values;
  ep.q_scales = (uint8_t*)q_scales;
  return dispatch<kEpiSwigluQuant>(a_values, a_scales, b_values, b_scales, ep, m, n, k, stream,
                                   "qia_mxfp8_gemm_swiglu_quant");
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

extern "C" int qia_mxfp8_gemm_grouped(int epilogue, const qia_mxfp8_gemm_problem* problems, int count, int64_t n,
                                      int64_t k, void* stream) {
  const char* who = "qia_mxfp8_gemm_grouped";
  if (!problems || count < 1 || count > 2) return set_error(QIA_ERR_INVALID, "%s: 1 or 2 problems", who);
  Problem pr[2];
  for (int i = 0; i < count; ++i) {
    const qia_mxfp8_gemm_problem& q = problems[i];
    if (q.bias && !aligned(q.bias, 16)) return set_error(QIA_ERR_ALIGNMENT, "%s: bias alignment", who);
    EpiParams ep{};
    ep.bias = (const __nv_bfloat16*)q.bias;
    if (epilogue == kEpiGeluQuant) {
      if (!q.q_values || !q.q_scales) return set_error(QIA_ERR_INVALID, "%s: null MXFP8 output", who);
      if (!aligned(q.q_values, 16)) return set_error(QIA_ERR_ALIGNMENT, "%s: output alignment", who);
      ep.q_values = (uint8_t*)q.q_values;
      ep.q_scales = (uint8_t*)q.q_scales;
    } else {
      int rc = check_out(q.out, q.ldo, n, who);
      if (rc) return rc;
      ep.out = (__nv_bfloat16*)q.out;
      ep.ldo = q.ldo;
    }
    if (epilogue == kEpiGateResidual) {
      if (!q.gate || !q.resid || q.rows_per_batch <= 0)
        return set_error(QIA_ERR_INVALID, "%s: gate/resid/rows_per_batch", who);
      if (!aligned(q.gate, 16) || !aligned(q.resid, 16)) return set_error(QIA_ERR_ALIGNMENT, "%s: alignment", who);
      ep.gate = (const __nv_bfloat16*)q.gate;
      ep.resid = (const __nv_bfloat16*)q.resid;
      ep.rows_per_batch = q.rows_per_batch;
    }
    pr[i] = Problem{q.a_values, q.a_scales, q.b_values, q.b_scales, ep, q.m};
  }
  switch (epilogue) {
    case kEpiBf16: return dispatch<kEpiBf16>(pr, count, n, k, stream, who);
    case kEpiGeluQuant: return dispatch<kEpiGeluQuant>(pr, count, n, k, stream, who);
    case kEpiGateResidual: return dispatch<kEpiGateResidual>(pr, count, n, k, stream, who);
    case kEpiGeluBf16: return dispatch<kEpiGeluBf16>(pr, count, n, k, stream, who);
    default: return set_error(QIA_ERR_INVALID, "%s: unknown epilogue %d", who, epilogue);
  }
}
