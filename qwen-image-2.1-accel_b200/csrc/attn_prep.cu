// Attention input preparation: per-head RMSNorm, complex RoPE and K/V packing.
//
// Numerics (reference src/qwen_image_accel/kernels/attention.py:44-77,
// kernels/bf16.py:46-55, kernels/elementwise.py:37-60):
//  * RMSNorm over head_dim (= 128): normalised value rounded to bf16, then the
//    product with the bf16 weight rounded to bf16 (Diffusers RMSNorm order).
//  * RoPE on interleaved pairs (re, im) with the CUDA complex multiply's FMA
//    order: re' = fma(re, c, -(im * s)), im' = fma(im, c, re * s), then bf16.
//
// Work split: one head row (128 bf16 = 256 B) per 16 threads, 8 contiguous
// elements (one 16-byte load) per thread; the sum of squares is a per-thread
// sum in PyTorch's mean(-1) order (see rms_normalize). RoPE pairs never cross a
// thread. Every access is a 16-byte vector access.
#include "qk_norm_rope.cuh"

namespace qia {
namespace {

using namespace qkrows;

__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                __nv_bfloat16* __restrict__ out, int64_t rows, float eps) {
  const int sub = threadIdx.x & (kLanesPerRow - 1);
  float wf[8];
  load_w(w, sub, wf);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x / kLanesPerRow;
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / kLanesPerRow; r < rows; r += stride) {
    float f[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(x + r * kHeadDim + sub * 8)), f);
    rms_normalize(f, wf, eps);
    *reinterpret_cast<uint4*>(out + r * kHeadDim + sub * 8) = pack8(f);
  }
}

__global__ void rope_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                            const float* __restrict__ freqs, __nv_bfloat16* __restrict__ oq,
                            __nv_bfloat16* __restrict__ ok, int64_t rows, int64_t seq, int64_t heads) {
  const int sub = threadIdx.x & (kLanesPerRow - 1);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x / kLanesPerRow;
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / kLanesPerRow; r < rows; r += stride) {
    const int64_t token = (r / heads) % seq;
    float cs[8];
    load_freqs(freqs, token, sub, cs);
    float f[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(q + r * kHeadDim + sub * 8)), f);
    rope8(f, cs);
    *reinterpret_cast<uint4*>(oq + r * kHeadDim + sub * 8) = pack8(f);
    unpack8(__ldg(reinterpret_cast<const uint4*>(k + r * kHeadDim + sub * 8)), f);
    rope8(f, cs);
    *reinterpret_cast<uint4*>(ok + r * kHeadDim + sub * 8) = pack8(f);
  }
}

// Units [0, target_rows) normalise+rotate q and k and copy v of one (b, s, h)
// row; units [target_rows, target_rows + prefix_rows) copy one cached (b, p, h)
// row of k and v to the front of the packed outputs.
__global__ void qknorm_rope_pack_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                        const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ ck,
                                        const __nv_bfloat16* __restrict__ cv, const __nv_bfloat16* __restrict__ wq,
                                        const __nv_bfloat16* __restrict__ wk, const float* __restrict__ freqs,
                                        __nv_bfloat16* __restrict__ oq, __nv_bfloat16* __restrict__ ok,
                                        __nv_bfloat16* __restrict__ ov, int64_t target_rows, int64_t prefix_rows,
                                        int64_t seq, int64_t prefix, int64_t heads, float eps_q, float eps_k) {
  const int sub = threadIdx.x & (kLanesPerRow - 1);
  float wqf[8], wkf[8];
  load_w(wq, sub, wqf);
  load_w(wk, sub, wkf);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x / kLanesPerRow;
  const int64_t total = target_rows + prefix_rows;
  for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / kLanesPerRow; u < total; u += stride) {
    if (u < target_rows) {
      const int64_t b = u / (seq * heads);
      const int64_t within = u - b * seq * heads;            // s * heads + h
      const int64_t token = within / heads;
      const int64_t dst = (b * (prefix + seq) * heads + prefix * heads + within) * kHeadDim + sub * 8;
      float cs[8];
      load_freqs(freqs, token, sub, cs);
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(q + u * kHeadDim + sub * 8)), f);
      rms_normalize(f, wqf, eps_q);
      rope8(f, cs);
      *reinterpret_cast<uint4*>(oq + u * kHeadDim + sub * 8) = pack8(f);
      unpack8(__ldg(reinterpret_cast<const uint4*>(k + u * kHeadDim + sub * 8)), f);
      rms_normalize(f, wkf, eps_k);
      rope8(f, cs);
      *reinterpret_cast<uint4*>(ok + dst) = pack8(f);
      *reinterpret_cast<uint4*>(ov + dst) = __ldg(reinterpret_cast<const uint4*>(v + u * kHeadDim + sub * 8));
    } else {
      const int64_t pu = u - target_rows;
      const int64_t b = pu / (prefix * heads);
      const int64_t within = pu - b * prefix * heads;
      const int64_t dst = (b * (prefix + seq) * heads + within) * kHeadDim + sub * 8;
      *reinterpret_cast<uint4*>(ok + dst) = __ldg(reinterpret_cast<const uint4*>(ck + pu * kHeadDim + sub * 8));
      *reinterpret_cast<uint4*>(ov + dst) = __ldg(reinterpret_cast<const uint4*>(cv + pu * kHeadDim + sub * 8));
    }
  }
}

// One segment of the joint [text, image] sequence from a fused q|k|v
// projection output with row stride ld_in.
__global__ void qknorm_rope_segment_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld_in,
                                           const __nv_bfloat16* __restrict__ wq,
                                           const __nv_bfloat16* __restrict__ wk, const float* __restrict__ freqs,
                                           __nv_bfloat16* __restrict__ oq, __nv_bfloat16* __restrict__ ok,
                                           __nv_bfloat16* __restrict__ ov, int64_t rows, int64_t seg_len,
                                           int64_t seq_offset, int64_t seq_total, int64_t heads, float eps_q,
                                           float eps_k) {
  const int sub = threadIdx.x & (kLanesPerRow - 1);
  float wqf[8], wkf[8];
  load_w(wq, sub, wqf);
  load_w(wk, sub, wkf);
  const int64_t qcols = heads * kHeadDim;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x / kLanesPerRow;
  for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / kLanesPerRow; u < rows; u += stride) {
    const int64_t h = u % heads;
    const int64_t tok = u / heads;           // b * seg_len + s
    const int64_t b = tok / seg_len;
    const int64_t s = tok - b * seg_len;
    const __nv_bfloat16* src = qkv + tok * ld_in + h * kHeadDim + sub * 8;
    const int64_t dst = ((b * seq_total + seq_offset + s) * heads + h) * kHeadDim + sub * 8;
    float cs[8];
    load_freqs(freqs, s, sub, cs);
    float f[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(src)), f);
    rms_normalize(f, wqf, eps_q);
    rope8(f, cs);
    *reinterpret_cast<uint4*>(oq + dst) = pack8(f);
    unpack8(__ldg(reinterpret_cast<const uint4*>(src + qcols)), f);
    rms_normalize(f, wkf, eps_k);
    rope8(f, cs);
    *reinterpret_cast<uint4*>(ok + dst) = pack8(f);
    *reinterpret_cast<uint4*>(ov + dst) = __ldg(reinterpret_cast<const uint4*>(src + 2 * qcols));
  }
}

unsigned grid_for(int64_t units, int threads) {
  const int64_t per_block = threads / kLanesPerRow;
  int64_t blocks = (units + per_block - 1) / per_block;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return unsigned(blocks);
}

bool al16(const void* p) { return p == nullptr || aligned(p, 16); }

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_rms_norm(const void* x, const void* weight, void* out, int64_t rows, int64_t dim, float eps,
                            void* stream) {
  if (!x || !weight || !out) return set_error(QIA_ERR_INVALID, "qia_rms_norm: null pointer");
  if (rows <= 0) return set_error(QIA_ERR_INVALID, "qia_rms_norm: rows=%lld", (long long)rows);
  if (dim != kHeadDim) return set_error(QIA_ERR_UNSUPPORTED, "qia_rms_norm: dim must be 128");
  if (!al16(x) || !al16(weight) || !al16(out)) return set_error(QIA_ERR_ALIGNMENT, "qia_rms_norm: 16-byte alignment");
  rms_norm_kernel<<<grid_for(rows, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (__nv_bfloat16*)out, rows, eps);
  return check_launch("rms_norm_kernel");
}

extern "C" int qia_rope_qk(const void* q, const void* k, const void* freqs, void* out_q, void* out_k,
                           int64_t batch, int64_t seq, int64_t heads, int64_t head_dim, void* stream) {
  if (!q || !k || !freqs || !out_q || !out_k) return set_error(QIA_ERR_INVALID, "qia_rope_qk: null pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0) return set_error(QIA_ERR_INVALID, "qia_rope_qk: bad sizes");
  if (head_dim != kHeadDim) return set_error(QIA_ERR_UNSUPPORTED, "qia_rope_qk: head_dim must be 128");
  if (!al16(q) || !al16(k) || !al16(freqs) || !al16(out_q) || !al16(out_k))
    return set_error(QIA_ERR_ALIGNMENT, "qia_rope_qk: 16-byte alignment");
  const int64_t rows = batch * seq * heads;
  rope_kernel<<<grid_for(rows, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const float*)freqs, (__nv_bfloat16*)out_q,
      (__nv_bfloat16*)out_k, rows, seq, heads);
  return check_launch("rope_kernel");
}

extern "C" int qia_qknorm_rope_pack(const void* q, const void* k, const void* v, const void* cached_k,
                                    const void* cached_v, const void* weight_q, const void* weight_k,
                                    const void* freqs, void* out_q, void* out_k, void* out_v, int64_t batch,
                                    int64_t seq, int64_t prefix, int64_t heads, int64_t head_dim, float eps_q,
                                    float eps_k, void* stream) {
  if (!q || !k || !v || !weight_q || !weight_k || !freqs || !out_q || !out_k || !out_v)
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_pack: null pointer");
  if (batch <= 0 || seq <= 0 || heads <= 0 || prefix < 0)
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_pack: bad sizes");
  if (prefix > 0 && (!cached_k || !cached_v))
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_pack: prefix > 0 needs cached k/v");
  if (head_dim != kHeadDim) return set_error(QIA_ERR_UNSUPPORTED, "qia_qknorm_rope_pack: head_dim must be 128");
  if (!al16(q) || !al16(k) || !al16(v) || !al16(cached_k) || !al16(cached_v) || !al16(weight_q) ||
      !al16(weight_k) || !al16(freqs) || !al16(out_q) || !al16(out_k) || !al16(out_v))
    return set_error(QIA_ERR_ALIGNMENT, "qia_qknorm_rope_pack: 16-byte alignment");
  const int64_t target = batch * seq * heads, pre = batch * prefix * heads;
  qknorm_rope_pack_kernel<<<grid_for(target + pre, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const __nv_bfloat16*)cached_k,
      (const __nv_bfloat16*)cached_v, (const __nv_bfloat16*)weight_q, (const __nv_bfloat16*)weight_k,
      (const float*)freqs, (__nv_bfloat16*)out_q, (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, target, pre, seq,
      prefix, heads, eps_q, eps_k);
  return check_launch("qknorm_rope_pack_kernel");
}

extern "C" int qia_qknorm_rope_segment(const void* qkv, int64_t ld_in, const void* weight_q, const void* weight_k,
                                       const void* freqs, void* out_q, void* out_k, void* out_v, int64_t batch,
                                       int64_t seg_len, int64_t seq_offset, int64_t seq_total, int64_t heads,
                                       int64_t head_dim, float eps_q, float eps_k, void* stream) {
  if (!qkv || !weight_q || !weight_k || !freqs || !out_q || !out_k || !out_v)
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_segment: null pointer");
  if (batch <= 0 || seg_len <= 0 || heads <= 0 || seq_offset < 0 || seq_offset + seg_len > seq_total)
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_segment: bad sizes");
  if (head_dim != kHeadDim) return set_error(QIA_ERR_UNSUPPORTED, "qia_qknorm_rope_segment: head_dim must be 128");
  if (ld_in < 3 * heads * head_dim || ld_in % 8 != 0)
    return set_error(QIA_ERR_INVALID, "qia_qknorm_rope_segment: ld_in=%lld too small or not a multiple of 8",
                     (long long)ld_in);
  if (!al16(qkv) || !al16(weight_q) || !al16(weight_k) || !al16(freqs) || !al16(out_q) || !al16(out_k) ||
      !al16(out_v))
    return set_error(QIA_ERR_ALIGNMENT, "qia_qknorm_rope_segment: 16-byte alignment");
  const int64_t rows = batch * seg_len * heads;
  qknorm_rope_segment_kernel<<<grid_for(rows, 256), 256, 0, as_stream(stream)>>>(
      (const __nv_bfloat16*)qkv, ld_in, (const __nv_bfloat16*)weight_q, (const __nv_bfloat16*)weight_k,
      (const float*)freqs, (__nv_bfloat16*)out_q, (__nv_bfloat16*)out_k, (__nv_bfloat16*)out_v, rows, seg_len,
      seq_offset, seq_total, heads, eps_q, eps_k);
  return check_launch("qknorm_rope_segment_kernel");
}
