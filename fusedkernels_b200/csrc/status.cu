// Status codes, per-thread error text and per-device attribute cache.
#include "common.cuh"

#include <mutex>

namespace fk {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return status;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FK_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return FK_OK;
}

int num_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace fk

extern "C" int fk_version(void) { return 100; }

extern "C" const char* fk_status_string(int status) {
  switch (status) {
    case FK_OK: return "ok";
    case FK_ERR_INVALID_ARG: return "invalid argument";
    case FK_ERR_UNSUPPORTED: return "unsupported shape";
    case FK_ERR_LAUNCH: return "kernel launch failed";
    case FK_ERR_WORKSPACE: return "workspace too small";
    case FK_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

extern "C" const char* fk_last_error(void) { return fk::g_err; }
