/*
 * qia_b200.h -- C ABI of the B200 (sm_100a) denoiser hot-path kernels.
 *
 * Every function takes plain device pointers, int64 sizes and the caller's
 * cudaStream_t (passed as void*), queues its kernel(s) on that stream and
 * returns a status code (QIA_OK == 0). No compute entry point allocates device
 * memory, synchronises the device or aborts the process (the qia_ipc_* set-up
 * entries of the multi-GPU exchange allocate, map and synchronise by design);
 * the text of the last failure on the calling host thread is returned by
 * qia_last_error_string().
 *
 * Tensor conventions (all contiguous unless a leading dimension is given):
 *   bf16       : __nv_bfloat16 / torch.bfloat16, row-major.
 *   MXFP8      : E4M3 codes [padded_rows, K] row-major plus E8M0 scales (one
 *                byte per 1x32 block along K) in the 128x4 blocked layout:
 *                byte((r, kb)) = ((r/128)*(K/128) + kb/4)*512 + (r%32)*16
 *                                + ((r/32)%4)*4 + kb%4,
 *                rows padded to a multiple of 128 (zeros in the padding).
 *   attention  : NHD, [batch, seq, heads, head_dim] bf16.
 *   RoPE freqs : complex64 viewed as float pairs, [seq, head_dim/2, 2] f32.
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the Qwen-Image-2.1-Accel checkout; WHL: = the pinned
 * diffusers wheel; SAGE: = the pinned SageAttention source).
 */
#ifndef QIA_B200_H_
#define QIA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum qia_status {
  QIA_OK = 0,
  QIA_ERR_INVALID = 1,      /* bad pointer, size, stride or argument */
  QIA_ERR_UNSUPPORTED = 2,  /* valid input outside what the kernel implements */
  QIA_ERR_ALIGNMENT = 3,    /* pointer or leading dimension misaligned */
  QIA_ERR_CUDA = 4,         /* a CUDA runtime call or launch failed */
  QIA_ERR_TIMEOUT = 5       /* a bounded device-side wait gave up */
};

/* Text of the last error raised on this host thread ("" if none). */
const char* qia_last_error_string(void);
/* ABI version: bumped whenever a signature changes. */
int qia_abi_version(void);

/* ---------------------------------------------------------------------------
 * Normalisation family
 * ------------------------------------------------------------------------ */

/* LayerNorm (no affine, eps) in PyTorch's CUDA Welford order, rounded to bf16,
 * times scale[b] (= 1 + s, bf16) -> bf16, plus optional shift[b] -> bf16.
 * x, out: [rows, dim]; scale, shift: [rows / rows_per_batch, dim]; shift may be
 * NULL. dim % 512 == 0, dim <= 8192.
 * Replaces: layer_norm_scale (src/qwen_image_accel/kernels/layernorm.py:58)
 * and the v1 img_norm1 + _modulate pair (WHL:diffusers/models/transformers/
 * transformer_qwenimage.py:683-717). */
int qia_ln_mod(const void* x, const void* scale, const void* shift, void* out,
               int64_t rows, int64_t dim, int64_t rows_per_batch, float eps,
               void* stream);

/* qia_ln_mod followed by MXFP8 quantization of the bf16 result, in one pass.
 * q_values: [padded_rows, dim] e4m3; q_scales: padded_rows*dim/32 bytes.
 * padded_rows = ceil(rows/128)*128; rows past `rows` are written as zeros.
 * Replaces: layer_norm_scale_quantize (src/qwen_image_accel/kernels/epilogue.py:76). */
int qia_ln_mod_quant(const void* x, const void* scale, const void* shift,
                     void* q_values, void* q_scales, int64_t rows, int64_t dim,
                     int64_t rows_per_batch, float eps, void* stream);

/* One qia_ln_mod_quant problem of a grouped launch. */
typedef struct qia_ln_mod_quant_problem {
  const void* x;           /* [rows, dim] bf16 */
  const void* scale;       /* [rows / rows_per_batch, dim] bf16 */
  const void* shift;       /* same shape, or NULL (all problems alike) */
  void* q_values;          /* [ceil(rows/128)*128, dim] e4m3 */
  void* q_scales;          /* blocked E8M0 */
  int64_t rows;
  int64_t rows_per_batch;
} qia_ln_mod_quant_problem;

/* One or two qia_ln_mod_quant problems with the same dim and eps in one
 * launch (count = 1 or 2): the dual-stream block's text rows (a few hundred)
 * run inside the image rows' launch instead of as a separate, latency-bound
 * launch. Each problem's outputs equal qia_ln_mod_quant's.
 * Replaces: the image- and text-stream layer_norm_scale_quantize pair
 * (src/qwen_image_accel/kernels/epilogue.py:76) of norm1 / norm2 of the v1
 * block (WHL:diffusers/models/transformers/transformer_qwenimage.py:683-717). */
int qia_ln_mod_quant_grouped(const qia_ln_mod_quant_problem* problems,
                             int count, int64_t dim, float eps, void* stream);

/* Gated residual: out = bf16(h + bf16(x * gate[b])). h, x, out: [rows, dim];
 * gate: [rows / rows_per_batch, dim].
 * Replaces: residual (src/qwen_image_accel/kernels/elementwise.py:26). */
int qia_gated_residual(const void* h, const void* x, const void* gate, void* out,
                       int64_t rows, int64_t dim, int64_t rows_per_batch,
                       void* stream);

/* The benchmark AdaLN composite (one pass):
 * out = bf16(r + bf16(gate * bf16(bf16(bf16(LN(x)) * scale) + shift))).
 * scale is the precomputed bf16 (1 + scale) vector, as in qia_ln_mod.
 * Replaces: the eager r + gate*(norm(x)*(1+scale)+shift) sequence of
 * WHL:diffusers/models/transformers/transformer_qwenimage.py:741-767. */
int qia_adaln_residual(const void* x, const void* r, const void* scale,
                       const void* shift, const void* gate, void* out,
                       int64_t rows, int64_t dim, int64_t rows_per_batch,
                       float eps, void* stream);

/* Per-row RMSNorm with bf16 weight, two bf16 rounding points
 * (normalised -> bf16, * weight -> bf16). x, out: [rows, dim], dim == 128.
 * Replaces: rms_norm (src/qwen_image_accel/kernels/bf16.py:58). */
int qia_rms_norm(const void* x, const void* weight, void* out, int64_t rows,
                 int64_t dim, float eps, void* stream);

/* AdaLN modulation vectors of one dual-stream block: out[r] =
 * bf16(W[r] . x + bias[r]) for the block's stacked img_mod / txt_mod linears
 * (weight [n, k] bf16, n = 12 * unit: each stream's shift1, scale1, gate1,
 * shift2, scale2, gate2 chunks of width unit), with the scale chunks (1 and 4
 * of every six) returned as bf16(1 + scale). x: SiLU(temb) [k] bf16. fp32
 * accumulation, one warp per output row. `ctas` bounds the grid: a small grid
 * (one CTA per SM) keeps the launch light enough to run beside the previous
 * block's kernels on another stream.
 * Replaces: img_mod / txt_mod Linear(SiLU(temb)) and the 1 + scale of
 * _modulate (WHL:diffusers/models/transformers/transformer_qwenimage.py:683-717). */
int qia_adaln_modulation(const void* x, const void* weight, const void* bias,
                         void* out, int64_t n, int64_t k, int64_t unit,
                         int64_t ctas, void* stream);

/* True-CFG combine with norm rescaling and the flow-match Euler update, one
 * launch: per row of dim channels, comb = neg + s*(cond - neg),
 * v = comb * (||cond|| / ||comb||), out = latents + dt * v, with every eager
 * bf16 boundary a bf16 rounding (fp32 sums of squares; the last add in fp32).
 * cond, neg, latents, out: [rows, dim] bf16 (out may be latents).
 * Replaces: the CFG combine of the v1 pipeline and the scheduler step
 * (WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
 * WHL:diffusers/schedulers/scheduling_flow_match_euler_discrete.py:483-517). */
int qia_cfg_euler(const void* cond, const void* neg, const void* latents,
                  void* out, int64_t rows, int64_t dim, float cfg_scale,
                  float dt, void* stream);

/* The Qwen-Image 2.1 joint-sequence RoPE table on the device: is_image
 * uint8 [seq] (1 = image token), block_hw HOST int32 [n_blocks, 2] (height,
 * width of each image block in sequence order, n_blocks <= 64), the three
 * per-axis complex64 tables (float pairs, rows_pos rows for positions 0.. then
 * rows_neg rows for positions -rows_neg..-1; pairs_* complex entries per row)
 * -> out complex64 [seq, pairs_frame + pairs_h + pairs_w]. Text tokens advance
 * one position on all axes; an image block freezes the frame axis and lays
 * its tokens on a centred height/width grid, then advances the position by
 * max(h, w). Bit-identical to the reference's table (an exact gather).
 * Replaces: QwenImage21Rope.forward's host loop and .tolist() sync
 * (WHL:diffusers/models/transformers/transformer_qwenimage21.py:677-710). */
int qia_rope21_table(const void* is_image, int64_t seq, const int32_t* block_hw,
                     int64_t n_blocks, const void* tab_frame, const void* tab_h,
                     const void* tab_w, int64_t pairs_frame, int64_t pairs_h,
                     int64_t pairs_w, int64_t rows_pos, int64_t rows_neg,
                     void* out, void* stream);

/* qia_cfg_euler with dt = sigmas[1] - sigmas[0] (fp32) read from device
 * memory (sigmas: device float[2] = {sigma, sigma_next}), so a step captured
 * in a CUDA graph replays with each step's schedule. Used by the CFG-split
 * (multi-GPU) step after the two halves' velocities are exchanged.
 * Replaces: the same reference sequence as qia_cfg_euler. */
int qia_cfg_euler_sched(const void* cond, const void* neg, const void* latents,
                        void* out, int64_t rows, int64_t dim, float cfg_scale,
                        const void* sigmas, void* stream);

/* The denoise step's tail as one tcgen05 kernel: proj_out of both CFG rows
 * (bf16 GEMM + bias, y bf16 [2*rows, k] row-major: rows [0, rows) the
 * conditional branch, [rows, 2*rows) the unconditional one; w bf16 [n, k];
 * bias bf16 [n] or NULL), the true-CFG combine with norm rescaling and the
 * Euler update into out [rows, n] (may be latents), with the roundings of
 * qia_cfg_euler; dt = sigmas[1] - sigmas[0] from device memory.
 * n must be 64 and k a multiple of 64; y, w, latents, out 16-byte aligned.
 * Replaces: proj_out + the CFG combine + FlowMatchEulerDiscreteScheduler.step
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:1007-1012;
 * WHL:diffusers/pipelines/qwenimage/pipeline_qwenimage.py:643-681;
 * WHL:diffusers/schedulers/scheduling_flow_match_euler_discrete.py:483-517). */
int qia_proj_out_cfg_euler(const void* y, const void* w, const void* bias,
                           const void* latents, void* out, int64_t rows,
                           int64_t k, int64_t n, float cfg_scale,
                           const void* sigmas, void* stream);

/* ---------------------------------------------------------------------------
 * Attention input preparation
 * ------------------------------------------------------------------------ */

/* Complex RoPE on interleaved pairs in the CUDA complex-FMA order.
 * q, k, out_q, out_k: [batch, seq, heads, head_dim]; freqs: [seq, head_dim/2, 2].
 * Replaces: rope_qk (src/qwen_image_accel/kernels/elementwise.py:63). */
int qia_rope_qk(const void* q, const void* k, const void* freqs, void* out_q,
                void* out_k, int64_t batch, int64_t seq, int64_t heads,
                int64_t head_dim, void* stream);

/* Q/K RMSNorm + RoPE + K/V pack after a cached prefix, one launch.
 * q, k, v: [batch, seq, heads, 128]; cached_k/v: [batch, prefix, heads, 128]
 * (may be NULL when prefix == 0); out_q: [batch, seq, heads, 128];
 * out_k/out_v: [batch, prefix + seq, heads, 128].
 * Replaces: prepare_attention_inputs (src/qwen_image_accel/kernels/attention.py:92). */
int qia_qknorm_rope_pack(const void* q, const void* k, const void* v,
                         const void* cached_k, const void* cached_v,
                         const void* weight_q, const void* weight_k,
                         const void* freqs, void* out_q, void* out_k,
                         void* out_v, int64_t batch, int64_t seq,
                         int64_t prefix, int64_t heads, int64_t head_dim,
                         float eps_q, float eps_k, void* stream);

/* Joint text+image variant for the dual-stream (v1) block: one segment of the
 * joint sequence. Reads q/k/v rows of this segment from a projection output
 * whose rows have leading dimension ld_in (elements; q at column 0, k at
 * q_cols, v at 2*q_cols where q_cols = heads*head_dim), applies RMSNorm with
 * this stream's weights and RoPE with this segment's freqs, and writes
 * [batch, seg_len] rows at sequence offset seq_offset of the joint
 * [batch, seq_total, heads, head_dim] outputs.
 * Replaces: the per-stream norm_q/norm_k/norm_added_q/norm_added_k + RoPE +
 * cat of QwenDoubleStreamAttnProcessor2_0
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:540-575). */
int qia_qknorm_rope_segment(const void* qkv, int64_t ld_in,
                            const void* weight_q, const void* weight_k,
                            const void* freqs, void* out_q, void* out_k,
                            void* out_v, int64_t batch, int64_t seg_len,
                            int64_t seq_offset, int64_t seq_total,
                            int64_t heads, int64_t head_dim, float eps_q,
                            float eps_k, void* stream);

/* ---------------------------------------------------------------------------
 * Feed-forward activations
 * ------------------------------------------------------------------------ */

/* SwiGLU: out = bf16(bf16(silu(gate)) * value), silu = div.rn(g, 1 + exp(-g)).
 * Replaces: swiglu (src/qwen_image_accel/kernels/bf16.py:27). */
int qia_swiglu(const void* gate, const void* value, void* out, int64_t n,
               void* stream);

/* SwiGLU + MXFP8 quantization. gate, value: [rows, width], width % 128 == 0.
 * Replaces: swiglu_quantize (src/qwen_image_accel/kernels/epilogue.py:123). */
int qia_swiglu_quant(const void* gate, const void* value, void* q_values,
                     void* q_scales, int64_t rows, int64_t width, void* stream);

/* GELU (tanh approximation, PyTorch CUDA formula) on bf16: out = bf16(gelu(x)).
 * Replaces: F.gelu(approximate="tanh") in the v1 FeedForward
 * (WHL:diffusers/models/activations.py:81-90). */
int qia_gelu_tanh(const void* x, void* out, int64_t n, void* stream);

/* ---------------------------------------------------------------------------
 * MXFP8 quantization
 * ------------------------------------------------------------------------ */

/* Quantize a bf16 [rows, k] matrix (row stride ld elements) to MXFP8.
 * k % 128 == 0. Outputs as described at the top of this file.
 * Replaces: quantize / _mx_quantize_kernel (src/qwen_image_accel/kernels/mxfp8.py:31-67). */
int qia_mxfp8_quantize(const void* x, int64_t ld, void* q_values, void* q_scales,
                       int64_t rows, int64_t k, void* stream);

/* ---------------------------------------------------------------------------
 * Block-scaled MXFP8 GEMM (tcgen05, TMEM accumulators, TMA-fed)
 *
 * A: MXFP8 activation [ceil(m/128)*128, k] + scales; B: MXFP8 weight [n, k]
 * (the nn.Linear weight layout) + scales; fp32 accumulation; bias: bf16 [n] or
 * NULL. k and n multiples of 128. Rows past m are not written (bf16 outputs).
 * Replaces: MXFP8Linear.matmul / torch._scaled_mm
 * (src/qwen_image_accel/optimizations/mxfp8.py:32-36), with the epilogues
 * of the dual-stream block's linears (WHL:diffusers/models/attention.py:1736,
 * activations.py:81-90, transformer_qwenimage.py:767-774).
 * ------------------------------------------------------------------------ */

/* out[m, n] (row stride ldo) = bf16(A . B^T + bias). */
int qia_mxfp8_gemm(const void* a_values, const void* a_scales, const void* b_values,
                   const void* b_scales, const void* bias, void* out, int64_t m,
                   int64_t n, int64_t k, int64_t ldo, void* stream);

/* out = bf16(gelu_tanh(bf16(A . B^T + bias))). */
int qia_mxfp8_gemm_gelu(const void* a_values, const void* a_scales,
                        const void* b_values, const void* b_scales,
                        const void* bias, void* out, int64_t m, int64_t n,
                        int64_t k, int64_t ldo, void* stream);

/* The FFN up-projection feeding the down-projection: the bf16 GELU result is
 * quantized to MXFP8 in the epilogue (n becomes the next GEMM's K).
 * q_values: [ceil(m/128)*128, n] e4m3 (padding rows zero), q_scales blocked. */
int qia_mxfp8_gemm_gelu_quant(const void* a_values, const void* a_scales,
                              const void* b_values, const void* b_scales,
                              const void* bias, void* q_values, void* q_scales,
                              int64_t m, int64_t n, int64_t k, void* stream);

/* The SwiGLU MLP's gate and value projections and the SwiGLU itself, one GEMM:
 * B stacks the two weights interleaved every 32 rows (rows [64 j, 64 j + 32)
 * = gate rows [32 j, 32 j + 32), the next 32 = value rows [32 j, 32 j + 32);
 * n = 2 * the MLP width, a multiple of 256). The epilogue rounds each gate and
 * value sum to bf16, forms bf16(silu(g) * v) with silu = bf16(g / (1 +
 * exp(-g))), and writes it as MXFP8 q_values [ceil(m/128)*128, n/2] + blocked
 * E8M0 q_scales (padding rows zero): byte-identical to qia_mxfp8_gemm of the
 * two projections followed by qia_swiglu_quant, without their bf16 outputs.
 * Replaces: _mx_mlp_forward's gate_layer.matmul + proj.matmul + swiglu_quantize
 * (src/qwen_image_accel/optimizations/quantized_decode.py:81-96). */
int qia_mxfp8_gemm_swiglu_quant(const void* a_values, const void* a_scales,
                                const void* b_values, const void* b_scales,
                                void* q_values, void* q_scales, int64_t m,
                                int64_t n, int64_t k, void* stream);

/* Gated residual epilogue: out = bf16(resid + bf16(gate[b] * bf16(A . B^T + bias)))
 * with b = row / rows_per_batch; gate: [m / rows_per_batch, n]; resid and out
 * share the row stride ldo and may be the same buffer (in-place update). */
int qia_mxfp8_gemm_gate_residual(const void* a_values, const void* a_scales,
                                 const void* b_values, const void* b_scales,
                                 const void* bias, const void* gate,
                                 const void* resid, void* out, int64_t m,
                                 int64_t n, int64_t k, int64_t ldo,
                                 int64_t rows_per_batch, void* stream);

/* One GEMM of a grouped launch. The fields an epilogue does not use are
 * ignored: out/ldo for QIA_EPI_GELU_QUANT, q_values/q_scales for the others,
 * gate/resid/rows_per_batch outside QIA_EPI_GATE_RESIDUAL. */
typedef struct qia_mxfp8_gemm_problem {
  const void* a_values;
  const void* a_scales;
  const void* b_values;
  const void* b_scales;
  const void* bias;       /* [n] bf16 or NULL */
  const void* gate;       /* [m / rows_per_batch, n] bf16 */
  const void* resid;      /* [m, ldo] bf16, may be out */
  void* out;              /* [m, ldo] bf16 */
  int64_t ldo;
  void* q_values;         /* [ceil(m/128)*128, n] e4m3 */
  void* q_scales;         /* blocked E8M0 */
  int64_t m;
  int64_t rows_per_batch;
} qia_mxfp8_gemm_problem;

enum qia_epilogue {
  QIA_EPI_BF16 = 0,          /* qia_mxfp8_gemm */
  QIA_EPI_GELU_QUANT = 1,    /* qia_mxfp8_gemm_gelu_quant */
  QIA_EPI_GATE_RESIDUAL = 2, /* qia_mxfp8_gemm_gate_residual */
  QIA_EPI_GELU_BF16 = 3      /* qia_mxfp8_gemm_gelu */
};

/* One or two GEMMs with the same n, k and epilogue in one persistent launch
 * (count = 1 or 2): output tiles of problem 0 first, then problem 1's, so a
 * small GEMM (the text stream's, m = batch * text tokens) fills the larger
 * one's last wave instead of running as a separate launch that leaves most
 * SMs idle. Each problem's results equal its single-GEMM entry point's.
 * Replaces: the image- and text-stream MXFP8Linear.matmul pair of each
 * projection of the dual-stream block (src/qwen_image_accel/optimizations/
 * mxfp8.py:32-36, called per stream by QwenDoubleStreamAttnProcessor2_0 and
 * the two MLPs, WHL:diffusers/models/transformers/transformer_qwenimage.py:
 * 540-600, 741-767). */
int qia_mxfp8_gemm_grouped(int epilogue, const qia_mxfp8_gemm_problem* problems,
                           int count, int64_t n, int64_t k, void* stream);

/* ---------------------------------------------------------------------------
 * Sage-style quantized attention (tcgen05: INT8 Q.K^T, FP8 P.V)
 *
 * q, k, v, out: bf16 [batch, seq, heads, 128] with element strides
 * (batch, seq, head) given per tensor in `strides` (q, k, v, out: 12 values;
 * the head_dim stride is 1). The caller provides a device workspace of
 * qia_sage_workspace_bytes() bytes (256-byte aligned) for the quantized
 * operands and their scales. sm_scale <= 0 selects 1/sqrt(head_dim).
 * Replaces: sage_decode / sageattn_qk_int8_pv_fp8_cuda(tensor_layout="NHD",
 * qk_quant_gran="per_warp", pv_accum_dtype="fp32+fp32")
 * (src/qwen_image_accel/optimizations/sage_attention.py:19-25;
 * SAGE:sageattention/core.py:636-828).
 * ------------------------------------------------------------------------ */
int64_t qia_sage_workspace_bytes(int64_t batch, int64_t heads, int64_t seq_q,
                                 int64_t seq_kv);

int qia_sage_attention(const void* q, const void* k, const void* v, void* out,
                       int64_t batch, int64_t seq_q, int64_t seq_kv,
                       int64_t heads, int64_t head_dim, const int64_t* strides,
                       float sm_scale, void* workspace, int64_t workspace_bytes,
                       void* stream);

/* Block-causal prefill: qia_sage_attention where query token t of batch b
 * attends to keys [0, kv_limit[b * kv_limit_stride_b + t]) only (int32,
 * clamped to [0, seq_kv]; kv_limit_stride_b 0 shares one row of limits across
 * the batch). The 2.1 prefill mask -- text tokens causal, every image block
 * bidirectional inside itself and causal towards what precedes it -- is one
 * such limit per query: t + 1 for a text token, the end of its image block
 * for an image token. Key tiles past a query tile's largest limit are not
 * visited. A row whose limit is 0 is written as zeros.
 * Replaces: the prefill branch of QwenImage21AttnProcessor (one SDPA call per
 * prefix segment plus one for the target image,
 * WHL:diffusers/models/transformers/transformer_qwenimage21.py:499-543) and
 * the flex_attention BlockMask of QwenImage21FlexAttnProcessor
 * (transformer_qwenimage21.py:257-306, 410-440). */
int qia_sage_attention_prefill(const void* q, const void* k, const void* v,
                               void* out, const int32_t* kv_limit,
                               int64_t kv_limit_stride_b, int64_t batch,
                               int64_t seq_q, int64_t seq_kv, int64_t heads,
                               int64_t head_dim, const int64_t* strides,
                               float sm_scale, void* workspace,
                               int64_t workspace_bytes, void* stream);

/* The joint [text, image] sequence written back as two streams: query tokens
 * [0, split) go to out_a ([batch, split, heads, 128]) and [split, seq_q) to
 * out_b ([batch, seq_q - split, heads, 128]); strides: q, k, v, out_a, out_b
 * (15 values). Replaces the joint attention + split of
 * QwenDoubleStreamAttnProcessor2_0
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:577-601). */
int qia_sage_attention_split(const void* q, const void* k, const void* v,
                             void* out_a, void* out_b, int64_t split,
                             int64_t batch, int64_t seq_q, int64_t seq_kv,
                             int64_t heads, int64_t head_dim,
                             const int64_t* strides, float sm_scale,
                             void* workspace, int64_t workspace_bytes,
                             void* stream);

/* qia_sage_attention_split with MXFP8 outputs: the two streams' attention
 * outputs bf16(O) are quantized in the attention epilogue to E4M3 rows
 * [batch * tokens, heads * 128] (a_*: query tokens [0, split), b_*: [split,
 * seq_q); rows padded to 128 are not written) with E8M0 scales in the 128x4
 * blocked layout -- byte-identical to qia_mxfp8_quantize of the bf16 outputs
 * and the A operand of the output-projection GEMMs (strides: q, k, v -- 9
 * values; values 32-byte, scales 4-byte aligned). split == seq_q gives one
 * stream: every query token goes to a_*, and b_values / b_scales may be null.
 * Replaces: the attention output -> MXFP8 quantize step of MXFusedProcessor
 * (src/qwen_image_accel/optimizations/quantized_decode.py:31-78). */
int qia_sage_attention_split_mx(const void* q, const void* k, const void* v,
                                void* a_values, void* a_scales,
                                void* b_values, void* b_scales, int64_t split,
                                int64_t batch, int64_t seq_q, int64_t seq_kv,
                                int64_t heads, int64_t head_dim,
                                const int64_t* strides, float sm_scale,
                                void* workspace, int64_t workspace_bytes,
                                void* stream);

/* The quantization half alone: Q INT8 per 32-token block, K mean-smoothed
 * INT8 per 64-token block, V FP8 per channel, written into the workspace
 * (strides: q, k, v -- 9 values).
 * Replaces: per_warp_int8 + per_channel_fp8 (SAGE:sageattention/quant.py). */
int qia_sage_quantize(const void* q, const void* k, const void* v,
                      int64_t batch, int64_t seq_q, int64_t seq_kv,
                      int64_t heads, int64_t head_dim, const int64_t* strides,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* qia_sage_quantize for the dual-stream block's joint [stream 0, stream 1]
 * sequence, reading Q/K/V straight from the two streams' fused q|k|v
 * projection outputs (rows b*len_i + s, leading dimension ld_i elements; q at
 * column 0, k at heads*128, v at 2*heads*128) and applying each stream's
 * per-head RMSNorm (weight_q_i / weight_k_i, eps) and RoPE (freqs_i: float32
 * [len_i, 64, 2]) on load, with the roundings of qia_qknorm_rope_segment: the
 * workspace is byte-identical to qia_qknorm_rope_segment on both streams
 * followed by qia_sage_quantize, without the bf16 Q/K/V in memory.
 * Replaces: the norm + RoPE + cat of QwenDoubleStreamAttnProcessor2_0
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:540-575) fused
 * with the quantization half of the reference's decode attention
 * (src/qwen_image_accel/optimizations/sage_attention.py:19-25). */
int qia_sage_quantize_joint(const void* qkv0, int64_t ld0, const void* qkv1,
                            int64_t ld1, const void* weight_q0,
                            const void* weight_k0, const void* weight_q1,
                            const void* weight_k1, const void* freqs0,
                            const void* freqs1, int64_t batch, int64_t len0,
                            int64_t len1, int64_t heads, int64_t head_dim,
                            float eps, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* qia_sage_quantize_joint followed by the attention with MXFP8 outputs per
 * stream (as qia_sage_attention_split_mx with split = len0): stream 0's rows
 * to a_values/a_scales, stream 1's to b_values/b_scales.
 * Replaces: the joint attention of QwenDoubleStreamAttnProcessor2_0
 * (WHL:diffusers/models/transformers/transformer_qwenimage.py:540-600) with
 * the reference's Sage decode attention
 * (src/qwen_image_accel/optimizations/quantized_decode.py:31-78). */
int qia_sage_attention_joint_mx(const void* qkv0, int64_t ld0, const void* qkv1,
                                int64_t ld1, const void* weight_q0,
                                const void* weight_k0, const void* weight_q1,
                                const void* weight_k1, const void* freqs0,
                                const void* freqs1, void* a_values,
                                void* a_scales, void* b_values, void* b_scales,
                                int64_t batch, int64_t len0, int64_t len1,
                                int64_t heads, int64_t head_dim, float eps,
                                float sm_scale, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* The attention half alone, on a workspace filled by qia_sage_quantize
 * (out_strides: 3 values).
 * Replaces: qk_int8_sv_f8_accum_f32_fuse_v_scale_attn_inst_buf
 * (SAGE:csrc/qattn/sm89_qk_int8_sv_f8_accum_f32_fuse_v_scale_attn_inst_buf.cu). */
int qia_sage_attn_quantized(const void* workspace, void* out, int64_t batch,
                            int64_t seq_q, int64_t seq_kv, int64_t heads,
                            int64_t head_dim, const int64_t* out_strides,
                            float sm_scale, void* stream);

/* ---- Ulysses exchanges over NVLink peer memory (CFG split x Ulysses) ----
 * The sharded dual-stream block moves each block's image q|k|v projection
 * rows from the rank that owns the tokens to the ranks that own the heads,
 * and the attention output back, by storing into the other ranks' device
 * buffers mapped with CUDA IPC. Each producing kernel's CTAs signal every
 * rank after their stores (system-scope fence, then a system-scope atomic add
 * on the receiving rank's 64-bit counter for this rank); qia_ulysses_wait
 * waits, with a time limit, for a round's signals.
 * Replaces: torch.distributed.all_to_all_single / all_gather under the
 * Ulysses helpers of the reference's dependency
 * (WHL:diffusers/models/attention_dispatch.py:2099-2182, 2510-2606). */

/* Size of an IPC handle (cudaIpcMemHandle_t). */
int64_t qia_ipc_handle_bytes(void);
/* A zeroed device buffer of `bytes` and its IPC handle (qia_ipc_handle_bytes
 * bytes at `handle`), for the other ranks to map. */
int qia_ipc_alloc(int64_t bytes, void** ptr, void* handle);
/* Map another process's buffer from its handle (peer access enabled lazily). */
int qia_ipc_open(const void* handle, void** ptr);
int qia_ipc_close(void* ptr);
int qia_ipc_free(void* ptr);

/* Rows s of this rank's fused q|k|v projection ([s_loc, ld] bf16: q, k, v of
 * `heads` heads of 128) -> every rank r's receive buffer recv_peers[r]
 * ([U * s_loc, 3 * (heads/U) * 128] bf16): row rank * s_loc + s, the q, k and
 * v of r's heads [r * heads/U, (r + 1) * heads/U) -- the layout
 * qia_sage_quantize_joint reads with heads/U heads. recv_peers and
 * signal_peers are device arrays of U pointers (this rank's own buffers at
 * index `rank`); the CTAs count themselves on `done` (uint64 in this rank's
 * memory, used by this entry only) and the launch's last CTA adds 1 to
 * signal_peers[r][rank] for every r. */
int qia_ulysses_scatter_qkv(const void* qkv, int64_t ld, int64_t s_loc,
                            int64_t heads, int64_t head_dim,
                            void* const* recv_peers, void* const* signal_peers,
                            void* done, int64_t ulysses, int64_t rank,
                            void* stream);
/* Wait for the next round of a wait site: *round (uint64, device, only this
 * entry updates it) += 1, then wait until counters[s] >= round * per_round
 * for s < sources. A wait longer than timeout_ns records QIA_ERR_TIMEOUT in
 * the device error word (qia_device_error) and returns. */
int qia_ulysses_wait(const void* counters, void* round, int64_t sources,
                     int64_t per_round, int64_t timeout_ns, void* stream);
/* CTAs of one unmasked attention launch (each signals every rank once in
 * qia_sage_attn_quantized_peers). */
int64_t qia_sage_attn_ctas(int64_t batch, int64_t heads, int64_t seq_q);
/* The attention half on a workspace filled by qia_sage_quantize_joint (batch
 * 1, `heads` heads, joint sequence of `seq` = split text + image tokens),
 * writing its output straight to the ranks that need it: image token j
 * (query split + j) to row j % peer_rows of img_peers[j / peer_rows], every
 * text token to each txt_peers[r], both [rows, heads_total * 128] bf16 at
 * head columns head0 .. head0 + heads - 1; then each CTA adds 1 to
 * signal_peers[r][slot] for every rank r. img_peers, txt_peers and
 * signal_peers are device arrays of peer_count pointers.
 * Replaces: the Ulysses attention's output all-to-all and the text all-gather
 * (WHL:diffusers/models/attention_dispatch.py:2510-2606) fused into the
 * reference's decode attention epilogue (src/qwen_image_accel/optimizations/
 * sage_attention.py:19-25). */
int qia_sage_attn_quantized_peers(const void* workspace, int64_t seq,
                                  int64_t heads, int64_t head_dim,
                                  int64_t split, void* const* img_peers,
                                  void* const* txt_peers, int64_t peer_rows,
                                  int64_t peer_count, int64_t head0,
                                  int64_t heads_total, void* const* signal_peers,
                                  int64_t slot, float sm_scale, void* stream);

/* Allocation-free variant of qia_sage_attention (no counterpart in the
 * reference): identical arguments minus the workspace. Some callers cannot
 * allocate device memory when they need attention -- a host that reaches the
 * GPU only through this C ABI (an FFI or plugin caller with no device
 * allocator of its own), a server whose device memory is a fixed pool owned
 * by another allocator, or a latency-critical loop that must not pay for
 * cudaMalloc/cudaFree, which synchronise the device. This entry point uses a
 * 16 MiB scratch array built into the library instead (held on every GPU
 * that loads the library until the process exits) and allocates nothing;
 * sizes whose workspace (qia_sage_workspace_bytes) exceeds 16 MiB are
 * rejected with QIA_ERR_UNSUPPORTED. The first call on each device looks up
 * the scratch's device address (make that first call before any stream
 * capture on that device). All calls share the one scratch array, whose
 * contents persist between calls: calls that may overlap on the GPU race. */
int qia_sage_attention_noalloc(const void* q, const void* k, const void* v,
                               void* out, int64_t batch, int64_t seq_q,
                               int64_t seq_kv, int64_t heads, int64_t head_dim,
                               const int64_t* strides, float sm_scale,
                               void* stream);

/* Reads and clears the device-side error word of the current device (set when
 * a bounded wait inside a tensor-core kernel gave up). Synchronises the device. */
int qia_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* QIA_B200_H_ */
