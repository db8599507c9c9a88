// Library-wide C-ABI helpers: version, error messages, wait bound, device check.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>

#include "b2m_host.h"

namespace b2m {

static thread_local char g_last_error[512] = {0};
static std::atomic<uint64_t> g_timeout_ns{2000000000ull};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B2M_OK;
  return fail(B2M_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

uint64_t timeout_ns() { return g_timeout_ns.load(std::memory_order_relaxed); }

int require_sm100(int* num_sms) {
  static std::mutex mu;
  static int cached_major[64] = {0};
  static int cached_sms[64] = {0};
  int dev = 0;
  B2M_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev < 0 || dev >= 64) return fail(B2M_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cached_major[dev] == 0) {
    cudaDeviceProp prop;
    B2M_TRY(check_cuda(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties"));
    cached_major[dev] = prop.major * 10 + prop.minor;
    cached_sms[dev] = prop.multiProcessorCount;
  }
  if (cached_major[dev] != 100)
    return fail(B2M_ERR_UNSUPPORTED, "b2m kernels need an sm_100 GPU (B200); device %d is sm_%d", dev,
                cached_major[dev]);
  if (num_sms) *num_sms = cached_sms[dev];
  return B2M_OK;
}

int driver_entry(const char* name, void** fn) {
  static std::mutex mu;
  static std::map<std::string, void*> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(name);
  if (it != cache.end()) {
    *fn = it->second;
    return B2M_OK;
  }
  cudaDriverEntryPointQueryResult q;
  void* p = nullptr;
  B2M_TRY(check_cuda(cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q), "cudaGetDriverEntryPoint"));
  if (q != cudaDriverEntryPointSuccess || !p) return fail(B2M_ERR_UNSUPPORTED, "%s not available from the driver", name);
  cache.emplace(name, p);
  *fn = p;
  return B2M_OK;
}

}  // namespace b2m

extern "C" {

int b2m_version(void) { return 100; }

const char* b2m_last_error(void) { return b2m::g_last_error; }

int b2m_set_timeout_ns(uint64_t ns) {
  if (ns < 1000000ull) return b2m::fail(B2M_ERR_ARG, "timeout %llu ns is below 1 ms", (unsigned long long)ns);
  b2m::g_timeout_ns.store(ns, std::memory_order_relaxed);
  return B2M_OK;
}

}  // extern "C"
