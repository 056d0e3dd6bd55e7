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

}  // namespace qia

extern "C" const char* qia_last_error_string(void) { return qia::g_last_error; }

extern "C" int qia_abi_version(void) { return 1; }
