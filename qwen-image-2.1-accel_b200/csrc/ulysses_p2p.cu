// Ulysses exchanges of the sharded dual-stream block over NVLink peer memory.
//
// The sequence-parallel joint attention (CFG split x Ulysses; the template the
// reference's dependency ships: WHL:diffusers/models/attention_dispatch.py:
// 2099-2182 all-to-all helpers, :2510-2606 Ulysses attention) moves, per
// block, the image tokens' q|k|v projection rows from the rank that owns the
// tokens to the ranks that own the heads, and the attention output back. Here
// both moves are stores into the other ranks' device buffers, mapped into
// every rank of the group with CUDA IPC (NVLink P2P): the q|k|v rows by
// ulysses_scatter_qkv_kernel below, the attention output by the attention
// kernel's own epilogue (sage_attn.cu, qia_sage_attn_quantized_peers).
//
// Completion protocol: every thread of a producing CTA issues a system-scope
// fence after its stores. The q|k|v producers (this scatter, or the QKV
// GEMM's scatter epilogue) then count their CTAs on a counter in this rank's
// memory, and the launch's last CTA adds 1 to every rank's 64-bit counter of
// this rank (a system-scope atomic through the peer mapping): one signal per
// launch, whichever producer ran. The attention signals from every CTA. The
// counters only grow, across calls and CUDA graph replays. The consuming
// rank's wait kernel keeps its own round number in device memory (so a
// replayed graph waits for the next round, not the one it was captured in)
// and waits, with a time limit, until every source's counter reaches round x
// (signals per round); on timeout it records QIA_ERR_TIMEOUT and returns.
// No TMA, no multicast, no library kernel touches peer memory.
#include <cstring>

#include "qia_common.cuh"
#include "sm100.cuh"

namespace qia {
namespace {

constexpr int kScatterThreads = 256;
constexpr int kHeadDim = 128;

struct ScatterArgs {
  const uint4* qkv;                    // [s_loc, ld] bf16 rows: q | k | v, `heads` heads of 128 each
  int64_t ld_chunks;                   // row stride in 16-byte chunks
  uint4* const* recv;                  // [U] each rank's receive buffer [U * s_loc, 3 * Hl * 128]
  unsigned long long* const* signal;   // [U] each rank's counters (this rank's slot u)
  unsigned long long* done;            // this rank's count of finished CTAs of this kernel
  int64_t s_loc;
  int heads, ulysses, u;
};

// Row s of this rank's tokens, piece (t, r) = head group r of section t (q, k
// or v), goes to rank r's receive row u * s_loc + s, section t. Consecutive
// threads copy consecutive 16-byte chunks of a source row, and a piece's
// chunks are contiguous at the destination.
__global__ void __launch_bounds__(kScatterThreads) ulysses_scatter_qkv_kernel(ScatterArgs a) {
  const int hl = a.heads / a.ulysses;
  const int piece = hl * (kHeadDim * 2 / 16);          // 16-byte chunks of one (section, head group)
  const int per_row = 3 * a.ulysses * piece;
  const int64_t total = a.s_loc * per_row;
  const int64_t dst_row0 = int64_t(a.u) * a.s_loc;
  for (int64_t i = int64_t(blockIdx.x) * kScatterThreads + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * kScatterThreads) {
    const int64_t row = i / per_row;
    const int rem = int(i - row * per_row);
    const int t = rem / (a.ulysses * piece);
    const int r = (rem / piece) % a.ulysses;
    const int c = rem % piece;
    const uint4 v = a.qkv[row * a.ld_chunks + rem];
    a.recv[r][(dst_row0 + row) * (3 * piece) + t * piece + c] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    // the launch's last CTA to finish signals every rank once
    const unsigned long long n = atomicAdd(a.done, 1ull) + 1ull;
    if (n % gridDim.x == 0) {
      __threadfence_system();
      for (int r = 0; r < a.ulysses; ++r) atomicAdd_system(a.signal[r] + a.u, 1ull);
    }
  }
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One thread: the next round of this wait site, then every source's counter.
__global__ void ulysses_wait_kernel(const unsigned long long* counters, unsigned long long* round, int sources,
                                    unsigned long long per_round, unsigned long long timeout_ns, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const unsigned long long r = *round + 1;
  *round = r;
  const unsigned long long want = r * per_round;
  const uint64_t t0 = global_timer_ns();
  for (int s = 0; s < sources; ++s) {
    while (ld_acquire_sys(counters + s) < want) {
      if (global_timer_ns() - t0 > timeout_ns) {
        if (err) atomicExch(err, QIA_ERR_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
  }
}

int scatter_grid(int64_t s_loc, int64_t heads) {
  const int64_t chunks = s_loc * 3 * heads * (kHeadDim * 2 / 16);
  const int64_t want = (chunks + kScatterThreads - 1) / kScatterThreads;
  const int64_t cap = int64_t(sm_count()) * 8;
  return int(want < cap ? want : cap);
}

}  // namespace
}  // namespace qia

using namespace qia;

extern "C" int64_t qia_ipc_handle_bytes(void) { return int64_t(sizeof(cudaIpcMemHandle_t)); }

extern "C" int qia_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  if (bytes <= 0 || !ptr || !handle) return set_error(QIA_ERR_INVALID, "qia_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, size_t(bytes));
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "qia_ipc_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, size_t(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(QIA_ERR_CUDA, "qia_ipc_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return QIA_OK;
}

extern "C" int qia_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return set_error(QIA_ERR_INVALID, "qia_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "qia_ipc_open: %s", cudaGetErrorString(e));
  return QIA_OK;
}

extern "C" int qia_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "qia_ipc_close: %s", cudaGetErrorString(e));
  return QIA_OK;
}

extern "C" int qia_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "qia_ipc_free: %s", cudaGetErrorString(e));
  return QIA_OK;
}

extern "C" int qia_ulysses_scatter_qkv(const void* qkv, int64_t ld, int64_t s_loc, int64_t heads, int64_t head_dim,
                                       void* const* recv_peers, void* const* signal_peers, void* done,
                                       int64_t ulysses, int64_t rank, void* stream) {
  if (!qkv || !recv_peers || !signal_peers || !done)
    return set_error(QIA_ERR_INVALID, "qia_ulysses_scatter_qkv: null pointer");
  if (!aligned(done, 8)) return set_error(QIA_ERR_ALIGNMENT, "qia_ulysses_scatter_qkv: done alignment");
  if (head_dim != kHeadDim) return set_error(QIA_ERR_UNSUPPORTED, "qia_ulysses_scatter_qkv: head_dim must be 128");
  if (s_loc <= 0 || heads <= 0 || ulysses <= 0 || ulysses > 64 || heads % ulysses || rank < 0 || rank >= ulysses)
    return set_error(QIA_ERR_INVALID, "qia_ulysses_scatter_qkv: s_loc=%lld heads=%lld U=%lld rank=%lld",
                     (long long)s_loc, (long long)heads, (long long)ulysses, (long long)rank);
  if (ld < 3 * heads * kHeadDim || ld % 8 || !aligned(qkv, 16))
    return set_error(QIA_ERR_ALIGNMENT, "qia_ulysses_scatter_qkv: rows must be >= 3*heads*128 wide, 16-byte aligned");
  ScatterArgs a;
  a.qkv = (const uint4*)qkv;
  a.ld_chunks = ld / 8;
  a.recv = (uint4* const*)recv_peers;
  a.signal = (unsigned long long* const*)signal_peers;
  a.done = (unsigned long long*)done;
  a.s_loc = s_loc;
  a.heads = int(heads);
  a.ulysses = int(ulysses);
  a.u = int(rank);
  ulysses_scatter_qkv_kernel<<<scatter_grid(s_loc, heads), kScatterThreads, 0, as_stream(stream)>>>(a);
  return check_launch("ulysses_scatter_qkv_kernel");
}

extern "C" int qia_ulysses_wait(const void* counters, void* round, int64_t sources, int64_t per_round,
                                int64_t timeout_ns, void* stream) {
  if (!counters || !round || sources <= 0 || sources > 64 || per_round <= 0 || timeout_ns <= 0)
    return set_error(QIA_ERR_INVALID, "qia_ulysses_wait: bad arguments");
  if (!aligned(counters, 8) || !aligned(round, 8))
    return set_error(QIA_ERR_ALIGNMENT, "qia_ulysses_wait: counters must be 8-byte aligned");
  ulysses_wait_kernel<<<1, 32, 0, as_stream(stream)>>>((const unsigned long long*)counters,
                                                       (unsigned long long*)round, int(sources),
                                                       (unsigned long long)per_round,
                                                       (unsigned long long)timeout_ns, device_error_word());
  return check_launch("ulysses_wait_kernel");
}
