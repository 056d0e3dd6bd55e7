/*
 * CPU oracle for the qia_* hot-path kernels -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic for the memory-bound
 * family and the MXFP8 quantizer. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg may load it, and only as the checker; the
 * product never links or calls it.
 *
 * Built with -ffp-contract=off: every fused multiply-add below is an explicit
 * fmaf(), every other operation rounds to fp32 on its own.
 *
 * Differences from the GPU that are known and bounded: rsqrtf/expf/tanhf are
 * computed here with correctly rounded (double precision) math, while the GPU
 * uses CUDA's rsqrtf/expf/tanhf, so a bf16 result can differ by one bf16 ulp
 * when the fp32 value sits at a rounding boundary. Integer outputs (MXFP8
 * codes and exponents) are exact functions of their bf16 inputs.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

/* ---------------------------------------------------------------- bf16 */
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f2bf(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rbf(float f) { return bf2f(f2bf(f)); }
static inline float f_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_f(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float rsqrt_ref(float x) { return (float)(1.0 / sqrt((double)x)); }

/* ---------------------------------------------------------------- E4M3 */
/* fp32 -> E4M3 (bias 7, max 448, no inf), round to nearest even, saturating
 * finite values to +-448 (cvt.rn.satfinite semantics). */
uint8_t oracle_e4m3(float x) {
  uint32_t u = bits_f(x);
  uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  float a = fabsf(x);
  if (isnan(x)) return (uint8_t)(sign | 0x7f);
  if (a >= 448.0f) return (uint8_t)(sign | 0x7e); /* 448 = 0x7e */
  /* smallest subnormal 2^-9; normal min 2^-6 */
  double v = (double)a;
  int e;
  double m = frexp(v, &e); /* v = m * 2^e, m in [0.5,1) */
  int exp_unbiased = e - 1; /* v = (2m) * 2^(e-1) */
  double quantum = exp_unbiased < -6 ? ldexp(1.0, -9) : ldexp(1.0, exp_unbiased - 3);
  if (v == 0.0) return sign;
  double q = v / quantum;
  double fl = floor(q);
  double rem = q - fl;
  double n = fl;
  if (rem > 0.5 || (rem == 0.5 && fmod(fl, 2.0) != 0.0)) n = fl + 1.0;
  double r = n * quantum;
  if (r > 448.0) r = 448.0;
  /* encode r */
  if (r == 0.0) return sign;
  if (r < ldexp(1.0, -6)) { /* subnormal: mantissa = r / 2^-9 */
    int mant = (int)(r / ldexp(1.0, -9));
    return (uint8_t)(sign | mant);
  }
  int re;
  double rm = frexp(r, &re);
  int be = re - 1 + 7;
  int mant = (int)((rm * 2.0 - 1.0) * 8.0 + 0.5);
  if (mant == 8) { mant = 0; be += 1; }
  return (uint8_t)(sign | (be << 3) | mant);
}

/* ---------------------------------------------------------------- MXFP8 */
/* reference src/qwen_image_accel/kernels/mxfp8.py:46-50 */
static inline int mx_exponent(float amax) {
  uint32_t b = bits_f(amax);
  int e = (int)((b >> 23) & 0xffu) - 8 + (((b & 0x7fffffu) > 6291456u) ? 1 : 0);
  if (e < 0) e = 0;
  if (e > 254) e = 254;
  return amax == 0.0f ? 0 : e;
}
/* reference src/qwen_image_accel/kernels/mxfp8.py:53-56 */
static inline int64_t mx_scale_offset(int64_t row, int64_t kb, int64_t kb_tiles) {
  return ((row >> 7) * kb_tiles + (kb >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (kb & 3);
}

/* Quantize one row block of 32 fp32 values (already bf16-representable). */
static void mx_block(const float* y, uint8_t* qv, uint8_t* qs, int64_t row, int64_t kb, int64_t k) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(y[i]));
  int e = mx_exponent(amax);
  float inv = f_bits((uint32_t)(254 - e) << 23);
  for (int i = 0; i < 32; ++i) qv[i] = oracle_e4m3(y[i] * inv);
  qs[mx_scale_offset(row, kb, k >> 7)] = (uint8_t)e;
}

/* reference src/qwen_image_accel/kernels/mxfp8.py:31-67 (rows padded to 128) */
void oracle_mx_quantize(const uint16_t* x, int64_t ld, uint8_t* qv, uint8_t* qs, int64_t rows, int64_t k) {
  int64_t padded = (rows + 127) / 128 * 128;
  float y[32];
  for (int64_t r = 0; r < padded; ++r)
    for (int64_t kb = 0; kb < k / 32; ++kb) {
      for (int i = 0; i < 32; ++i) y[i] = r < rows ? bf2f(x[r * ld + kb * 32 + i]) : 0.0f;
      mx_block(y, qv + r * k + kb * 32, qs, r, kb, k);
    }
}

/* ---------------------------------------------------------------- LayerNorm */
typedef struct { float mean, m2, count; } welford_t;

/* cuWelfordCombine(dataB = own, dataA = other) */
static welford_t combine(welford_t own, welford_t other) {
  welford_t r;
  float delta = own.mean - other.mean;
  float count = other.count + own.count;
  float coef = 1.0f / count;
  float na = other.count * coef, nb = own.count * coef;
  r.mean = fmaf(na, other.mean, nb * own.mean);
  r.m2 = fmaf((delta * delta) * other.count, nb, other.m2 + own.m2);
  r.count = count;
  return r;
}

/* Row statistics in PyTorch 2.11's vectorised CUDA LayerNorm order
 * (reference src/qwen_image_accel/kernels/layernorm.py:17-47, generalised from
 * dim = 4096 to any dim % 512 == 0): 128 lanes, lane t owns the vec4 groups
 * t*4 + j*512; shuffle-down merges 16..1 inside each warp; warp 0 += warp 2,
 * warp 1 += warp 3, then warp 0 += warp 1. */
void oracle_ln_stats(const uint16_t* xrow, int dim, float* mean_out, float* var_out) {
  welford_t lane[128], next[128];
  int nv = dim / 512;
  for (int t = 0; t < 128; ++t) {
    float mean = 0.0f, m2 = 0.0f;
    for (int j = 0; j < nv; ++j)
      for (int ii = 0; ii < 4; ++ii) {
        float x = bf2f(xrow[t * 4 + j * 512 + ii]);
        float inv = 1.0f / (float)(j * 4 + ii + 1);
        float delta = x - mean;
        mean = fmaf(delta, inv, mean);
        m2 = fmaf(delta, x - mean, m2);
      }
    lane[t].mean = mean;
    lane[t].m2 = m2;
    lane[t].count = (float)(nv * 4);
  }
  for (int off = 16; off > 0; off >>= 1) {
    for (int t = 0; t < 128; ++t) {
      int w = t >> 5, l = t & 31;
      welford_t other = (l + off < 32) ? lane[w * 32 + l + off] : lane[t];
      next[t] = combine(lane[t], other);
    }
    memcpy(lane, next, sizeof(lane));
  }
  welford_t w0 = combine(lane[0], lane[64]);
  welford_t w1 = combine(lane[32], lane[96]);
  w0 = combine(w0, w1);
  *mean_out = w0.mean;
  *var_out = w0.m2 / (float)dim;
}

/* LN -> bf16 -> * scale -> bf16 [-> + shift -> bf16]
 * reference kernels/layernorm.py:48-55 and the v1 _modulate
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:683-717) */
static void ln_mod_row(const uint16_t* xrow, const uint16_t* scale, const uint16_t* shift, int dim, float eps,
                       float* y) {
  float mean, var;
  oracle_ln_stats(xrow, dim, &mean, &var);
  float rstd = rsqrt_ref(var + eps);
  for (int c = 0; c < dim; ++c) {
    float nrm = rbf(rstd * (bf2f(xrow[c]) - mean));
    float m = rbf(nrm * bf2f(scale[c]));
    if (shift) m = rbf(m + bf2f(shift[c]));
    y[c] = m;
  }
}

void oracle_ln_mod(const uint16_t* x, const uint16_t* scale, const uint16_t* shift, uint16_t* out, int64_t rows,
                   int dim, int64_t rows_per_batch, float eps) {
  float* y = (float*)malloc(sizeof(float) * dim);
  for (int64_t r = 0; r < rows; ++r) {
    int64_t b = r / rows_per_batch;
    ln_mod_row(x + r * dim, scale + b * dim, shift ? shift + b * dim : NULL, dim, eps, y);
    for (int c = 0; c < dim; ++c) out[r * dim + c] = f2bf(y[c]);
  }
  free(y);
}

/* reference kernels/epilogue.py:24-73: LN-mod then the quantizer on the bf16 result */
void oracle_ln_mod_quant(const uint16_t* x, const uint16_t* scale, const uint16_t* shift, uint8_t* qv, uint8_t* qs,
                         int64_t rows, int dim, int64_t rows_per_batch, float eps) {
  int64_t padded = (rows + 127) / 128 * 128;
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * rows * dim);
  oracle_ln_mod(x, scale, shift, tmp, rows, dim, rows_per_batch, eps);
  oracle_mx_quantize(tmp, dim, qv, qs, rows, dim);
  (void)padded;
  free(tmp);
}

/* r + gate * (LN(x) * scale + shift), each eager op rounded to bf16 */
void oracle_adaln_residual(const uint16_t* x, const uint16_t* r, const uint16_t* scale, const uint16_t* shift,
                           const uint16_t* gate, uint16_t* out, int64_t rows, int dim, int64_t rows_per_batch,
                           float eps) {
  float* y = (float*)malloc(sizeof(float) * dim);
  for (int64_t i = 0; i < rows; ++i) {
    int64_t b = i / rows_per_batch;
    ln_mod_row(x + i * dim, scale + b * dim, shift + b * dim, dim, eps, y);
    for (int c = 0; c < dim; ++c)
      out[i * dim + c] = f2bf(bf2f(r[i * dim + c]) + rbf(bf2f(gate[b * dim + c]) * y[c]));
  }
  free(y);
}

/* reference kernels/elementwise.py:10-23: h + bf16(x * gate) */
void oracle_gated_residual(const uint16_t* h, const uint16_t* x, const uint16_t* gate, uint16_t* out, int64_t rows,
                           int64_t dim, int64_t rows_per_batch) {
  for (int64_t i = 0; i < rows; ++i) {
    int64_t b = i / rows_per_batch;
    for (int64_t c = 0; c < dim; ++c)
      out[i * dim + c] = f2bf(bf2f(h[i * dim + c]) + rbf(bf2f(x[i * dim + c]) * bf2f(gate[b * dim + c])));
  }
}

/* ---------------------------------------------------------------- QK norm + RoPE */
/* reference kernels/bf16.py:46-55 (RMSNorm, two rounding points). The sum of
 * squares follows PyTorch's CUDA mean(-1) over 128 fp32 values (the eager
 * Diffusers RMSNorm), checked against torch on the GPU: 32 vec4 partials
 * ((a+b)+c)+d over contiguous groups, then a halving tree g[t] += g[t + w]
 * for w = 16, 8, 4, 2, 1. Squares of bf16 values are exact in fp32. */
static void rms_row(const float* in, const uint16_t* w, float eps, float* out) {
  float part[32];
  for (int t = 0; t < 32; ++t) {
    const float* e = in + 4 * t;
    part[t] = ((e[0] * e[0] + e[1] * e[1]) + e[2] * e[2]) + e[3] * e[3];
  }
  for (int width = 16; width >= 1; width >>= 1)
    for (int t = 0; t < width; ++t) part[t] = part[t] + part[t + width];
  float r = rsqrt_ref(part[0] / 128.0f + eps);
  for (int c = 0; c < 128; ++c) out[c] = rbf(rbf(in[c] * r) * bf2f(w[c]));
}

/* reference kernels/elementwise.py:48-56 / attention.py:62-73 */
static void rope_row(float* f, const float* cs) {
  for (int p = 0; p < 64; ++p) {
    float re = f[2 * p], im = f[2 * p + 1], c = cs[2 * p], s = cs[2 * p + 1];
    f[2 * p] = fmaf(re, c, -(im * s));
    f[2 * p + 1] = fmaf(im, c, re * s);
  }
}

void oracle_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* out, int64_t rows, float eps) {
  float in[128], o[128];
  for (int64_t r = 0; r < rows; ++r) {
    for (int c = 0; c < 128; ++c) in[c] = bf2f(x[r * 128 + c]);
    rms_row(in, w, eps, o);
    for (int c = 0; c < 128; ++c) out[r * 128 + c] = f2bf(o[c]);
  }
}

void oracle_rope_qk(const uint16_t* q, const uint16_t* k, const float* freqs, uint16_t* oq, uint16_t* ok,
                    int64_t batch, int64_t seq, int64_t heads) {
  float f[128];
  for (int64_t r = 0; r < batch * seq * heads; ++r) {
    int64_t tok = (r / heads) % seq;
    for (int c = 0; c < 128; ++c) f[c] = bf2f(q[r * 128 + c]);
    rope_row(f, freqs + tok * 128);
    for (int c = 0; c < 128; ++c) oq[r * 128 + c] = f2bf(f[c]);
    for (int c = 0; c < 128; ++c) f[c] = bf2f(k[r * 128 + c]);
    rope_row(f, freqs + tok * 128);
    for (int c = 0; c < 128; ++c) ok[r * 128 + c] = f2bf(f[c]);
  }
}

/* reference kernels/attention.py:16-89 (prepare_attention_inputs) */
void oracle_qknorm_rope_pack(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* ck,
                             const uint16_t* cv, const uint16_t* wq, const uint16_t* wk, const float* freqs,
                             uint16_t* oq, uint16_t* ok, uint16_t* ov, int64_t batch, int64_t seq, int64_t prefix,
                             int64_t heads, float eps_q, float eps_k) {
  float in[128], o[128];
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t p = 0; p < prefix; ++p)
      for (int64_t h = 0; h < heads; ++h) {
        int64_t src = ((b * prefix + p) * heads + h) * 128;
        int64_t dst = ((b * (prefix + seq) + p) * heads + h) * 128;
        memcpy(ok + dst, ck + src, 256);
        memcpy(ov + dst, cv + src, 256);
      }
    for (int64_t s = 0; s < seq; ++s)
      for (int64_t h = 0; h < heads; ++h) {
        int64_t src = ((b * seq + s) * heads + h) * 128;
        int64_t dst = ((b * (prefix + seq) + prefix + s) * heads + h) * 128;
        for (int c = 0; c < 128; ++c) in[c] = bf2f(q[src + c]);
        rms_row(in, wq, eps_q, o);
        rope_row(o, freqs + s * 128);
        for (int c = 0; c < 128; ++c) oq[src + c] = f2bf(o[c]);
        for (int c = 0; c < 128; ++c) in[c] = bf2f(k[src + c]);
        rms_row(in, wk, eps_k, o);
        rope_row(o, freqs + s * 128);
        for (int c = 0; c < 128; ++c) ok[dst + c] = f2bf(o[c]);
        memcpy(ov + dst, v + src, 256);
      }
  }
}

/* One segment of the v1 joint [text, image] sequence
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:540-575). */
void oracle_qknorm_rope_segment(const uint16_t* qkv, int64_t ld_in, const uint16_t* wq, const uint16_t* wk,
                                const float* freqs, uint16_t* oq, uint16_t* ok, uint16_t* ov, int64_t batch,
                                int64_t seg_len, int64_t seq_offset, int64_t seq_total, int64_t heads, float eps_q,
                                float eps_k) {
  float in[128], o[128];
  int64_t qcols = heads * 128;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t s = 0; s < seg_len; ++s)
      for (int64_t h = 0; h < heads; ++h) {
        const uint16_t* src = qkv + (b * seg_len + s) * ld_in + h * 128;
        int64_t dst = ((b * seq_total + seq_offset + s) * heads + h) * 128;
        for (int c = 0; c < 128; ++c) in[c] = bf2f(src[c]);
        rms_row(in, wq, eps_q, o);
        rope_row(o, freqs + s * 128);
        for (int c = 0; c < 128; ++c) oq[dst + c] = f2bf(o[c]);
        for (int c = 0; c < 128; ++c) in[c] = bf2f(src[qcols + c]);
        rms_row(in, wk, eps_k, o);
        rope_row(o, freqs + s * 128);
        for (int c = 0; c < 128; ++c) ok[dst + c] = f2bf(o[c]);
        memcpy(ov + dst, src + 2 * qcols, 256);
      }
}

/* ---------------------------------------------------------------- FFN */
/* reference kernels/bf16.py:12-24: bf16(div.rn(g, 1 + exp(-g))) * v */
static inline float silu_ref(float g) { return rbf(g / (1.0f + (float)exp(-(double)g))); }

void oracle_swiglu(const uint16_t* g, const uint16_t* v, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(silu_ref(bf2f(g[i])) * bf2f(v[i]));
}

/* reference kernels/epilogue.py:96-120 */
void oracle_swiglu_quant(const uint16_t* g, const uint16_t* v, uint8_t* qv, uint8_t* qs, int64_t rows,
                         int64_t width) {
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * rows * width);
  oracle_swiglu(g, v, tmp, rows * width);
  oracle_mx_quantize(tmp, width, qv, qs, rows, width);
  free(tmp);
}

/* PyTorch CUDA GELU (approximate='tanh') in fp32 opmath */
static inline float gelu_tanh_ref(float x) {
  const float k_beta = (float)(M_SQRT2 * M_2_SQRTPI * 0.5);
  const float k_kappa = 0.044715f;
  float x_cube = (x * x) * x;
  float inner = k_beta * fmaf(k_kappa, x_cube, x);
  return (0.5f * x) * (1.0f + (float)tanh((double)inner));
}

float oracle_gelu_tanh_f32(float x) { return gelu_tanh_ref(x); }

void oracle_gelu_tanh(const uint16_t* x, uint16_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(gelu_tanh_ref(bf2f(x[i])));
}
