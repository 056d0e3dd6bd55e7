// Error reporting and small host utilities shared by every qia_* entry point.
#include "qia_common.cuh"

#include <mutex>

namespace qia {

namespace {
thread_local char g_last_error[512] = {0};
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(QIA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return QIA_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

__device__ int g_qia_device_error = 0;

int* device_error_word() {
  static int* cached[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qia_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

}  // namespace qia

extern "C" int qia_device_error(int* code) {
  if (!code) return qia::set_error(QIA_ERR_INVALID, "qia_device_error: null output");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, qia::g_qia_device_error, sizeof(int));
  if (e != cudaSuccess) return qia::set_error(QIA_ERR_CUDA, "qia_device_error: %s", cudaGetErrorString(e));
  const int zero = 0;
  e = cudaMemcpyToSymbol(qia::g_qia_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return qia::set_error(QIA_ERR_CUDA, "qia_device_error: %s", cudaGetErrorString(e));
  *code = v;
  return QIA_OK;
}

extern "C" const char* qia_last_error_string(void) { return qia::g_last_error; }

extern "C" int qia_abi_version(void) { return 1; }
