// The Qwen-Image 2.1 joint-sequence RoPE table built on the device.
//
// Reference: QwenImage21Rope.forward (WHL:diffusers/models/transformers/
// transformer_qwenimage21.py:677-710), a host loop over the sequence with a
// .tolist() of the image mask every forward. Its integer positions, per token
// t of the joint sequence:
//   * text tokens advance one shared position on all three axes (frame,
//     height, width all = the position);
//   * image blocks are taken in order from img_shapes, block b covering the
//     h_b * w_b image tokens that follow the previous block; a block freezes
//     the frame axis at the position the preceding text reached, lays its
//     tokens out row-major on a height/width grid centred on zero
//     (height index  i / w_b - (h_b - h_b / 2), width index i % w_b - (w_b -
//     w_b / 2) for its i-th token), then advances the position by
//     max(h_b, w_b).
// Closed form used here: for token t, with T(t) the text tokens before t and
// I(t) the image tokens before t,
//   frame(t) = T(t) + sum_{b' < b} max(h_b', w_b')
// where b is t's block (image token) or the number of blocks whose tokens all
// precede t (text token). The table row is then the per-axis complex64 rows
// at those positions (a negative position p indexes row rows_axis + p, as the
// reference's negative indexing does), concatenated: the gather is exact, so
// the table is bit-identical to the reference's.
//
// Launch: one thread per token; every CTA first counts the text tokens of
// the mask before its own range (its threads stride over that prefix), then
// scans its own 256 tokens.
#include "qia_common.cuh"

namespace qia {
namespace {

constexpr int kRtThreads = 256;
constexpr int kRtMaxBlocks = 64;

struct RopeTableParams {
  const uint8_t* is_image;    // [S] 1 = image token
  int hw[kRtMaxBlocks][2];    // (height, width) of each image block, sequence order
  int n_blocks;
  const float2* tab[3];       // per axis complex64 [rows_axis, pairs_axis]
  int pairs[3];               // 8, 28, 28 for axes 16/56/56
  int rows_axis;              // rows of each axis table: rows_pos non-negative positions, then rows_neg
  float2* out;                // [S, pairs0 + pairs1 + pairs2]
  int64_t S;
};

__device__ __forceinline__ int block_sum_exclusive(int v, int* scratch, int* total) {
  // exclusive prefix sum over the CTA (256 threads), warp shuffles then warp totals
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kRtThreads / 32 ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kRtThreads / 32) scratch[lane] = w;     // inclusive warp totals
  }
  __syncthreads();
  const int before = (warp ? scratch[warp - 1] : 0) + x - v;
  if (total) *total = scratch[kRtThreads / 32 - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kRtThreads) rope21_table_kernel(RopeTableParams p, int* err) {
  __shared__ int scratch[kRtThreads / 32];
  __shared__ int s_hw[kRtMaxBlocks][2];
  __shared__ int s_cum_tokens[kRtMaxBlocks + 1];   // image tokens before block b
  __shared__ int s_cum_adv[kRtMaxBlocks + 1];      // sum of max(h, w) over blocks before b
  const int64_t t0 = int64_t(blockIdx.x) * kRtThreads;
  const int64_t t = t0 + threadIdx.x;
  if (threadIdx.x == 0) {
    int ct = 0, ca = 0;
    for (int b = 0; b < p.n_blocks; ++b) {
      const int h = p.hw[b][0], w = p.hw[b][1];
      s_hw[b][0] = h;
      s_hw[b][1] = w;
      s_cum_tokens[b] = ct;
      s_cum_adv[b] = ca;
      ct += h * w;
      ca += h > w ? h : w;
    }
    s_cum_tokens[p.n_blocks] = ct;
    s_cum_adv[p.n_blocks] = ca;
  }
  // image tokens in [0, t0): every thread counts a strided share of the prefix
  int img_prefix = 0;
  for (int64_t i = threadIdx.x; i < t0; i += kRtThreads) img_prefix += p.is_image[i] ? 1 : 0;
  int prefix_total = 0;
  block_sum_exclusive(img_prefix, scratch, &prefix_total);
  const bool live = t < p.S;
  const int img = live && p.is_image[t] ? 1 : 0;
  const int img_before = prefix_total + block_sum_exclusive(img, scratch, nullptr);
  if (!live) return;
  const int text_before = int(t) - img_before;
  // the block of image-rank j = img_before (image token) or the count of
  // blocks completed before t (text token)
  int b = 0;
  while (b < p.n_blocks && s_cum_tokens[b + 1] <= img_before) ++b;
  const int frame = text_before + s_cum_adv[b];
  int hpos = frame, wpos = frame;
  if (img && b < p.n_blocks) {
    const int i = img_before - s_cum_tokens[b];
    const int h = s_hw[b][0], w = s_hw[b][1];
    hpos = i / w - (h - h / 2);
    wpos = i % w - (w - w / 2);
  }
  const int pos[3] = {frame, hpos, wpos};
  float2* dst = p.out + t * int64_t(p.pairs[0] + p.pairs[1] + p.pairs[2]);
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const int row = pos[a] >= 0 ? pos[a] : p.rows_axis + pos[a];
    if (row < 0 || row >= p.rows_axis) {
      // only a mask with more text tokens than img_shapes accounts for gets
      // here (the host bounds the consistent case): no read, zeros, an error
      if (err) atomicExch(err, QIA_ERR_INVALID);
      for (int c = 0; c < p.pairs[a]; ++c) dst[c] = make_float2(0.0f, 0.0f);
    } else {
      const float2* src = p.tab[a] + int64_t(row) * p.pairs[a];
      for (int c = 0; c < p.pairs[a]; ++c) dst[c] = src[c];
    }
    dst += p.pairs[a];
  }
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int qia_rope21_table(const void* is_image, int64_t seq, const int32_t* block_hw, int64_t n_blocks,
                                const void* tab_frame, const void* tab_h, const void* tab_w, int64_t pairs_frame,
                                int64_t pairs_h, int64_t pairs_w, int64_t rows_pos, int64_t rows_neg, void* out,
                                void* stream) {
  if (!is_image || (n_blocks && !block_hw) || !tab_frame || !tab_h || !tab_w || !out)
    return set_error(QIA_ERR_INVALID, "qia_rope21_table: null pointer");
  if (seq <= 0 || seq > (int64_t(1) << 30) || n_blocks < 0 || n_blocks > kRtMaxBlocks)
    return set_error(QIA_ERR_INVALID, "qia_rope21_table: seq=%lld n_blocks=%lld", (long long)seq,
                     (long long)n_blocks);
  if (pairs_frame <= 0 || pairs_h <= 0 || pairs_w <= 0 || rows_pos <= 0 || rows_neg < 0 ||
      rows_pos + rows_neg > (int64_t(1) << 30))
    return set_error(QIA_ERR_INVALID, "qia_rope21_table: bad table sizes");
  if (!aligned(tab_frame, 8) || !aligned(tab_h, 8) || !aligned(tab_w, 8) || !aligned(out, 8))
    return set_error(QIA_ERR_ALIGNMENT, "qia_rope21_table: misaligned pointer");
  RopeTableParams p;
  // every position must index a row: with the mask holding the sum(h * w)
  // image tokens img_shapes accounts for, frame <= (seq - sum h*w) + sum
  // max(h, w) (text and block advances) < rows_pos; grid offsets in
  // [-(n - n/2), n/2) within both halves. (A mask inconsistent with the
  // shapes is caught on the device: see the kernel.)
  int64_t reach = seq, tokens = 0;
  for (int64_t b = 0; b < n_blocks; ++b) {
    const int64_t h = block_hw[2 * b], w = block_hw[2 * b + 1];
    if (h <= 0 || w <= 0 || h > 65536 || w > 65536)
      return set_error(QIA_ERR_INVALID, "qia_rope21_table: block %lld is %lld x %lld", (long long)b, (long long)h,
                       (long long)w);
    if (h - h / 2 > rows_neg || w - w / 2 > rows_neg || h / 2 > rows_pos || w / 2 > rows_pos)
      return set_error(QIA_ERR_UNSUPPORTED, "qia_rope21_table: a %lld x %lld grid exceeds the tables",
                       (long long)h, (long long)w);
    reach += h > w ? h : w;
    tokens += h * w;
    p.hw[b][0] = int(h);
    p.hw[b][1] = int(w);
  }
  if (tokens > seq)
    return set_error(QIA_ERR_INVALID, "qia_rope21_table: img_shapes hold %lld tokens, the sequence %lld",
                     (long long)tokens, (long long)seq);
  reach -= tokens;
  if (reach > rows_pos)
    return set_error(QIA_ERR_UNSUPPORTED, "qia_rope21_table: positions reach %lld, tables hold %lld",
                     (long long)reach, (long long)rows_pos);
  p.is_image = (const uint8_t*)is_image;
  p.n_blocks = int(n_blocks);
  p.tab[0] = (const float2*)tab_frame;
  p.tab[1] = (const float2*)tab_h;
  p.tab[2] = (const float2*)tab_w;
  p.pairs[0] = int(pairs_frame);
  p.pairs[1] = int(pairs_h);
  p.pairs[2] = int(pairs_w);
  p.rows_axis = int(rows_pos + rows_neg);
  p.out = (float2*)out;
  p.S = seq;
  const int64_t grid = (seq + kRtThreads - 1) / kRtThreads;
  rope21_table_kernel<<<unsigned(grid), kRtThreads, 0, as_stream(stream)>>>(p, device_error_word());
  return check_launch("rope21_table_kernel");
}
