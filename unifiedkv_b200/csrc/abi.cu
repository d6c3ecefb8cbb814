// Error state, device queries and version of libbpkv.so.
#include <stdarg.h>
#include <mutex>

#include "common.cuh"

namespace bpkv {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace bpkv

extern "C" BPKV_API const char* bpkv_last_error(void) { return bpkv::g_err; }

extern "C" BPKV_API int bpkv_version(void) { return 200; }

#ifndef BPKV_BUILD_HASH
#define BPKV_BUILD_HASH "unstamped"
#endif
// Hash of the sources this library was built from (unifiedkv_b200/build.py, tree_hash).
extern "C" BPKV_API const char* bpkv_build_hash(void) { return BPKV_BUILD_HASH; }

extern "C" BPKV_API int bpkv_num_sms(void) { return bpkv::sm_count(); }
