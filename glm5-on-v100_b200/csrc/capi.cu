// Status plumbing of the C ABI: thread-local error text, device queries.
#include "common.cuh"

namespace dsa {

namespace {
thread_local std::string g_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 0;
  return d;
}

int sm_count(int dev) {
  static int cache[kMaxDevices] = {0};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace dsa

extern "C" const char* dsa_last_error(void) { return dsa::g_last_error.c_str(); }

extern "C" int dsa_version(void) { return (1 << 16) | 0; }
