// Library-wide host state: per-thread error message, SM-count cache, version.
#include "common.cuh"

#include <mutex>
#include <string.h>

namespace ml {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int num_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) dev = 0;
  if (dev >= 64) dev = 63;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace ml

extern "C" int ml_version(void) { return 100; /* 0.1.0 */ }

extern "C" const char* ml_last_error(void) { return ml::g_last_error; }
