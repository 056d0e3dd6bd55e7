// LayerNorm + AdaLN modulation family and the gated residual.
//
// Numerics follow the reference contracts:
//  * LayerNorm statistics in PyTorch 2.11's vectorised CUDA LayerNorm order
//    (reference src/qwen_image_accel/kernels/layernorm.py:17-55): 128 threads
//    per row, each owning the vec4 groups t*4 + j*512 (j < dim/512) and running
//    one Welford update per element; then five shuffle-down merges inside each
//    warp and the warp 0+2, 0+1 merges through shared memory, each merge in
//    cuWelfordCombine's arithmetic; var = m2 / dim, rstd = rsqrtf(var + eps).
//  * Every eager bf16 tensor boundary is kept as a bf16 rounding point
//    (normalised, *scale, +shift, *gate, +residual).
//  * The MXFP8 epilogue quantizes the bf16 result exactly as the standalone
//    quantizer does (reference kernels/epilogue.py:24-73).
//
// HBM layout: rows are contiguous [rows, dim] bf16; one 128-thread CTA per row
// keeps the row in registers (dim/128 fp32 per thread), so x is read once.
#include "qia_common.cuh"

namespace qia {
namespace {

constexpr int kThreads = 128;
enum Mode { kModBf16 = 0, kModQuant = 1, kAdalnResidual = 2 };

struct Welford {
  float mean, m2, count;
};

// cuWelfordCombine(dataB = own, dataA = other) as PyTorch's warp and block
// reductions use it -- delta = own.mean - other.mean, coef = 1/count,
// mean = fma(other.count*coef, other.mean, own.count*coef * own.mean),
// m2 = fma(delta^2 * other.count, own.count*coef, other.m2 + own.m2) -- for two
// partials over the same known number of elements CNT (every merge of the
// row reduction pairs equal counts: 4*NV per thread, doubling with each
// merge), so the count-only terms (1/count and count*coef, both correctly
// rounded) are folded at compile time.
template <int CNT>
__device__ __forceinline__ Welford welford_combine_eq(const Welford own, const Welford other) {
  constexpr float count = float(2 * CNT);
  constexpr float coef = 1.0f / count;
  constexpr float n_ab = float(CNT) * coef;
  const float delta = own.mean - other.mean;
  Welford r;
  r.mean = __fmaf_rn(n_ab, other.mean, __fmul_rn(n_ab, own.mean));
  r.m2 = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), float(CNT)), n_ab, other.m2 + own.m2);
  r.count = count;
  return r;
}

template <int NV, int LEVEL>
__device__ __forceinline__ Welford shuffle_merges(Welford w) {
  // five shuffle-down merges (offsets 16, 8, 4, 2, 1); partial counts 4*NV * 2^LEVEL
  if constexpr (LEVEL < 5) {
    Welford o;
    o.mean = __shfl_down_sync(0xffffffffu, w.mean, 16 >> LEVEL);
    o.m2 = __shfl_down_sync(0xffffffffu, w.m2, 16 >> LEVEL);
    o.count = w.count;
    return shuffle_merges<NV, LEVEL + 1>(welford_combine_eq<(4 * NV) << LEVEL>(w, o));
  } else {
    return w;
  }
}

template <int NV>
__device__ __forceinline__ void row_stats(const __nv_bfloat16* __restrict__ xrow, bool live,
                                          float (&v)[NV * 4], float& mean, float& rstd,
                                          int dim, float eps) {
  __shared__ float s_stat[4];
  const int t = threadIdx.x;
  uint2 raw[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    raw[j] = live ? __ldg(reinterpret_cast<const uint2*>(xrow + t * 4 + j * 512)) : make_uint2(0u, 0u);
  }
  Welford w{0.0f, 0.0f, float(NV * 4)};
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    unpack4(raw[j], &v[j * 4]);
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const float inv = 1.0f / float(j * 4 + ii + 1);
      const float x = v[j * 4 + ii];
      const float delta = x - w.mean;
      w.mean = __fmaf_rn(delta, inv, w.mean);
      w.m2 = __fmaf_rn(delta, x - w.mean, w.m2);
    }
  }
  w = shuffle_merges<NV, 0>(w);
  __shared__ Welford s_w[2];
  const int warp = t >> 5, lane = t & 31;
  // upper half of the warps hands its partial to the lower half (offset 2, then 1)
  if (lane == 0 && warp >= 2) s_w[warp - 2] = w;
  __syncthreads();
  if (lane == 0 && warp < 2) w = welford_combine_eq<(4 * NV) << 5>(w, s_w[warp]);
  __syncthreads();
  if (lane == 0 && warp == 1) s_w[0] = w;
  __syncthreads();
  if (t == 0) {
    w = welford_combine_eq<(4 * NV) << 6>(w, s_w[0]);
    s_stat[0] = w.mean;
    s_stat[1] = __fdiv_rn(w.m2, float(dim));
  }
  __syncthreads();
  mean = s_stat[0];
  rstd = rsqrtf(s_stat[1] + eps);
}

// The arguments of one LayerNorm problem; a launch may hold two (the dual-
// stream block's image and text rows): CTAs [0, split) take problem 0's rows,
// the rest problem 1's, so the small text problem rides in the image launch.
struct LnArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* resid;
  const __nv_bfloat16* scale;
  const __nv_bfloat16* shift;
  const __nv_bfloat16* gate;
  __nv_bfloat16* out;
  uint8_t* q_values;
  uint8_t* q_scales;
  int64_t rows;
  int rows_per_batch;
};

template <int NV, int MODE, bool SHIFT>
__global__ void __launch_bounds__(kThreads)
ln_mod_kernel(const LnArgs a0, const LnArgs a1, int64_t split, float eps) {
  constexpr int D = NV * 512;
  const bool second = blockIdx.x >= split;
  const LnArgs& a = second ? a1 : a0;
  const __nv_bfloat16* __restrict__ x = a.x;
  const __nv_bfloat16* __restrict__ resid = a.resid;
  const __nv_bfloat16* __restrict__ scale = a.scale;
  const __nv_bfloat16* __restrict__ shift = a.shift;
  const __nv_bfloat16* __restrict__ gate = a.gate;
  __nv_bfloat16* __restrict__ out = a.out;
  uint8_t* __restrict__ q_values = a.q_values;
  uint8_t* __restrict__ q_scales = a.q_scales;
  const int64_t rows = a.rows;
  const int rows_per_batch = a.rows_per_batch;
  const int64_t row = second ? int64_t(blockIdx.x) - split : int64_t(blockIdx.x);
  const bool live = row < rows;
  const int t = threadIdx.x;
  float v[NV * 4];
  float mean, rstd;
  row_stats<NV>(x + row * D, live, v, mean, rstd, D, eps);

  const int64_t vec_row = live ? (row / rows_per_batch) * D : 0;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = t * 4 + j * 512;
    // bf16(rstd * (x - mean)), then bf16(. * scale) and bf16(. + shift): the
    // operands of the last two are bf16 values, so the packed bf16x2 multiply
    // and add (one rounding each) give the fp32-then-round results
    const uint2 s2 = __ldg(reinterpret_cast<const uint2*>(scale + vec_row + c));
    uint32_t y01 = cvt_bf16x2(__fmul_rn(rstd, v[j * 4] - mean), __fmul_rn(rstd, v[j * 4 + 1] - mean));
    uint32_t y23 = cvt_bf16x2(__fmul_rn(rstd, v[j * 4 + 2] - mean), __fmul_rn(rstd, v[j * 4 + 3] - mean));
    y01 = mul_bf16x2(y01, s2.x);
    y23 = mul_bf16x2(y23, s2.y);
    if (SHIFT) {
      const uint2 h2 = __ldg(reinterpret_cast<const uint2*>(shift + vec_row + c));
      y01 = add_bf16x2(y01, h2.x);
      y23 = add_bf16x2(y23, h2.y);
    }
    if (!live) y01 = y23 = 0u;
    if (MODE == kModBf16) {
      *reinterpret_cast<uint2*>(out + row * D + c) = make_uint2(y01, y23);
    } else if (MODE == kAdalnResidual) {
      // r + bf16(gate * y), rounded: both steps on bf16 operands
      const uint2 g2 = __ldg(reinterpret_cast<const uint2*>(gate + vec_row + c));
      const uint2 r2 = __ldg(reinterpret_cast<const uint2*>(resid + row * D + c));
      *reinterpret_cast<uint2*>(out + row * D + c) =
          make_uint2(add_bf16x2(r2.x, mul_bf16x2(g2.x, y01)), add_bf16x2(r2.y, mul_bf16x2(g2.y, y23)));
    } else {
      // 32-element MX block = 8 consecutive threads (aligned groups of 8 lanes)
      const uint32_t m2 = max_bf16x2(abs_bf16x2(y01), abs_bf16x2(y23));
      float amax = fmaxf(bf16_lo(m2), bf16_hi(m2));
      amax = warp_max_xor(amax, 4);
      const int e = mx_exponent(amax);
      const float inv = mx_inverse_scale(e);
      const uint32_t codes =
          cvt_e4m3x4(bf16_lo(y01) * inv, bf16_hi(y01) * inv, bf16_lo(y23) * inv, bf16_hi(y23) * inv);
      *reinterpret_cast<uint32_t*>(q_values + row * D + c) = codes;
      if ((t & 7) == 0) q_scales[mx_scale_offset(row, c >> 5, D / 128)] = uint8_t(e);
    }
  }
}

// grid0 (grid1) CTAs for problem 0 (1): its rows, or its rows padded to 128
// for the MXFP8 output.
template <int MODE, bool SHIFT>
int launch_ln(int nv, cudaStream_t st, const LnArgs& a0, int64_t grid0, const LnArgs& a1, int64_t grid1,
              float eps) {
  const dim3 grid{unsigned(grid0 + grid1)};
#define QIA_LN_CASE(N)                                                             \
  case N:                                                                          \
    ln_mod_kernel<N, MODE, SHIFT><<<grid, kThreads, 0, st>>>(a0, a1, grid0, eps);  \
    break;
  switch (nv) {
    QIA_LN_CASE(1) QIA_LN_CASE(2) QIA_LN_CASE(3) QIA_LN_CASE(4) QIA_LN_CASE(5) QIA_LN_CASE(6)
    QIA_LN_CASE(7) QIA_LN_CASE(8) QIA_LN_CASE(9) QIA_LN_CASE(10) QIA_LN_CASE(11) QIA_LN_CASE(12)
    QIA_LN_CASE(13) QIA_LN_CASE(14) QIA_LN_CASE(15) QIA_LN_CASE(16)
    default:
      return set_error(QIA_ERR_UNSUPPORTED, "layer norm: dim/512 = %d outside [1, 16]", nv);
  }
#undef QIA_LN_CASE
  return check_launch("ln_mod_kernel");
}

LnArgs ln_args(const void* x, const void* resid, const void* scale, const void* shift, const void* gate, void* out,
               void* qv, void* qs, int64_t rows, int64_t rows_per_batch) {
  LnArgs a;
  a.x = (const __nv_bfloat16*)x;
  a.resid = (const __nv_bfloat16*)resid;
  a.scale = (const __nv_bfloat16*)scale;
  a.shift = (const __nv_bfloat16*)shift;
  a.gate = (const __nv_bfloat16*)gate;
  a.out = (__nv_bfloat16*)out;
  a.q_values = (uint8_t*)qv;
  a.q_scales = (uint8_t*)qs;
  a.rows = rows;
  a.rows_per_batch = int(rows_per_batch);
  return a;
}

int validate_ln(const void* x, const void* scale, const void* out, int64_t rows, int64_t dim,
                int64_t rows_per_batch, const char* who) {
  if (!x || !scale || !out) return set_error(QIA_ERR_INVALID, "%s: null pointer", who);
  if (rows <= 0 || dim <= 0 || rows_per_batch <= 0)
    return set_error(QIA_ERR_INVALID, "%s: rows=%lld dim=%lld rows_per_batch=%lld", who, (long long)rows,
                     (long long)dim, (long long)rows_per_batch);
  if (dim % 512 != 0 || dim > 8192)
    return set_error(QIA_ERR_UNSUPPORTED, "%s: dim=%lld must be a multiple of 512 and <= 8192", who,
                     (long long)dim);
  if (rows > 0x7fffffffLL) return set_error(QIA_ERR_UNSUPPORTED, "%s: too many rows", who);
  if (!aligned(x, 8) || !aligned(scale, 8) || !aligned(out, 8))
    return set_error(QIA_ERR_ALIGNMENT, "%s: pointers must be 8-byte aligned", who);
  return QIA_OK;
}

// ---------------------------------------------------------------------------
// gated residual: out = bf16(h + bf16(x * gate))
// ---------------------------------------------------------------------------
__global__ void gated_residual_kernel(const uint4* __restrict__ h, const uint4* __restrict__ x,
                                      const __nv_bfloat16* __restrict__ gate, uint4* __restrict__ out,
                                      int64_t n8, int64_t dim, int64_t batch_elems) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t c = e % dim;
    const int64_t b = e / batch_elems;
    float fh[8], fx[8], fg[8], o[8];
    unpack8(__ldg(h + i), fh);
    unpack8(__ldg(x + i), fx);
    unpack8(__ldg(reinterpret_cast<const uint4*>(gate + b * dim + c)), fg);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = __fadd_rn(fh[k], round_bf16(__fmul_rn(fx[k], fg[k])));
    out[i] = pack8(o);
  }
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_ln_mod(const void* x, const void* scale, const void* shift, void* out, int64_t rows,
                          int64_t dim, int64_t rows_per_batch, float eps, void* stream) {
  int rc = validate_ln(x, scale, out, rows, dim, rows_per_batch, "qia_ln_mod");
  if (rc) return rc;
  if (shift && !aligned(shift, 8)) return set_error(QIA_ERR_ALIGNMENT, "qia_ln_mod: shift misaligned");
  const int nv = int(dim / 512);
  const LnArgs a = ln_args(x, nullptr, scale, shift, nullptr, out, nullptr, nullptr, rows, rows_per_batch);
  if (shift) return launch_ln<kModBf16, true>(nv, as_stream(stream), a, rows, a, 0, eps);
  return launch_ln<kModBf16, false>(nv, as_stream(stream), a, rows, a, 0, eps);
}

extern "C" int qia_ln_mod_quant(const void* x, const void* scale, const void* shift, void* q_values,
                                void* q_scales, int64_t rows, int64_t dim, int64_t rows_per_batch, float eps,
                                void* stream) {
  int rc = validate_ln(x, scale, q_values, rows, dim, rows_per_batch, "qia_ln_mod_quant");
  if (rc) return rc;
  if (!q_scales) return set_error(QIA_ERR_INVALID, "qia_ln_mod_quant: null q_scales");
  if (shift && !aligned(shift, 8)) return set_error(QIA_ERR_ALIGNMENT, "qia_ln_mod_quant: shift misaligned");
  const int64_t padded = (rows + 127) / 128 * 128;
  const int nv = int(dim / 512);
  const LnArgs a = ln_args(x, nullptr, scale, shift, nullptr, nullptr, q_values, q_scales, rows, rows_per_batch);
  if (shift) return launch_ln<kModQuant, true>(nv, as_stream(stream), a, padded, a, 0, eps);
  return launch_ln<kModQuant, false>(nv, as_stream(stream), a, padded, a, 0, eps);
}

extern "C" int qia_ln_mod_quant_grouped(const qia_ln_mod_quant_problem* problems, int count, int64_t dim,
                                        float eps, void* stream) {
  const char* who = "qia_ln_mod_quant_grouped";
  if (!problems || count < 1 || count > 2) return set_error(QIA_ERR_INVALID, "%s: 1 or 2 problems", who);
  LnArgs a[2];
  int64_t grid[2] = {0, 0};
  const bool shift = problems[0].shift != nullptr;
  for (int i = 0; i < count; ++i) {
    const qia_ln_mod_quant_problem& p = problems[i];
    int rc = validate_ln(p.x, p.scale, p.q_values, p.rows, dim, p.rows_per_batch, who);
    if (rc) return rc;
    if (!p.q_scales) return set_error(QIA_ERR_INVALID, "%s: null q_scales", who);
    if ((p.shift != nullptr) != shift) return set_error(QIA_ERR_INVALID, "%s: shift on some problems only", who);
    if (p.shift && !aligned(p.shift, 8)) return set_error(QIA_ERR_ALIGNMENT, "%s: shift misaligned", who);
    a[i] = ln_args(p.x, nullptr, p.scale, p.shift, nullptr, nullptr, p.q_values, p.q_scales, p.rows,
                   p.rows_per_batch);
    grid[i] = (p.rows + 127) / 128 * 128;
  }
  if (grid[0] + grid[1] > 0x7fffffffLL) return set_error(QIA_ERR_UNSUPPORTED, "%s: too many rows", who);
  if (count == 1) a[1] = a[0];
  const int nv = int(dim / 512);
  if (shift) return launch_ln<kModQuant, true>(nv, as_stream(stream), a[0], grid[0], a[1], grid[1], eps);
  return launch_ln<kModQuant, false>(nv, as_stream(stream), a[0], grid[0], a[1], grid[1], eps);
}

extern "C" int qia_adaln_residual(const void* x, const void* r, const void* scale, const void* shift,
                                  const void* gate, void* out, int64_t rows, int64_t dim, int64_t rows_per_batch,
                                  float eps, void* stream) {
  int rc = validate_ln(x, scale, out, rows, dim, rows_per_batch, "qia_adaln_residual");
  if (rc) return rc;
  if (!r || !shift || !gate) return set_error(QIA_ERR_INVALID, "qia_adaln_residual: null r/shift/gate");
  if (!aligned(r, 8) || !aligned(shift, 8) || !aligned(gate, 8))
    return set_error(QIA_ERR_ALIGNMENT, "qia_adaln_residual: pointers must be 8-byte aligned");
  const int nv = int(dim / 512);
  const LnArgs a = ln_args(x, r, scale, shift, gate, out, nullptr, nullptr, rows, rows_per_batch);
  return launch_ln<kAdalnResidual, true>(nv, as_stream(stream), a, rows, a, 0, eps);
}

extern "C" int qia_gated_residual(const void* h, const void* x, const void* gate, void* out, int64_t rows,
                                  int64_t dim, int64_t rows_per_batch, void* stream) {
  if (!h || !x || !gate || !out) return set_error(QIA_ERR_INVALID, "qia_gated_residual: null pointer");
  if (rows <= 0 || dim <= 0 || rows_per_batch <= 0)
    return set_error(QIA_ERR_INVALID, "qia_gated_residual: bad sizes");
  if (dim % 8 != 0) return set_error(QIA_ERR_UNSUPPORTED, "qia_gated_residual: dim %% 8 != 0");
  if (!aligned(h, 16) || !aligned(x, 16) || !aligned(gate, 16) || !aligned(out, 16))
    return set_error(QIA_ERR_ALIGNMENT, "qia_gated_residual: pointers must be 16-byte aligned");
  const int64_t n8 = rows * dim / 8;
  const int threads = 256;
  int64_t blocks = (n8 + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  gated_residual_kernel<<<unsigned(blocks), threads, 0, as_stream(stream)>>>(
      (const uint4*)h, (const uint4*)x, (const __nv_bfloat16*)gate, (uint4*)out, n8, dim, rows_per_batch * dim);
  return check_launch("gated_residual_kernel");
}
