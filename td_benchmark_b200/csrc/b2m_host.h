// Host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b2m.h"

namespace b2m {

// Record a formatted message for b2m_last_error() and return `code`.
int fail(int code, const char* fmt, ...);

// B2M_OK if `e` is cudaSuccess, otherwise B2M_ERR_CUDA with the CUDA message.
int check_cuda(cudaError_t e, const char* what);

// Process-wide bound for device spin waits (ns).
uint64_t timeout_ns();

// B2M_OK when the current device is sm_100 (cached per device).
int require_sm100(int* num_sms);

// Driver API entry point by name, resolved once per process (thread-safe).  The CUDA
// runtime is linked statically, so driver calls it does not wrap are reached this way.
int driver_entry(const char* name, void** fn);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace b2m

#define B2M_TRY(expr)              \
  do {                             \
    int _rc = (expr);              \
    if (_rc != B2M_OK) return _rc; \
  } while (0)
