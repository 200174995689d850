// Shared helpers for the libgq kernels: status plumbing, launch checks,
// bounded device-side waits and small warp utilities.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <cstdarg>

#include "../../include/gq.h"

namespace gq {

// Per-thread last error message, returned by gq_last_error().
void set_error(const char* fmt, ...);
const char* last_error();

inline int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return status;
}

// Count of kernels this library has launched (every launch site calls
// check_launch right after the launch); read with gq_launch_count().
void note_launch();

inline int check_launch(const char* what) {
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(GQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return GQ_OK;
}

#define GQ_CHECK_CUDA(call)                                                   \
  do {                                                                        \
    cudaError_t _e = (call);                                                  \
    if (_e != cudaSuccess)                                                    \
      return ::gq::fail(GQ_ECUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call,  \
                        cudaGetErrorString(_e));                              \
  } while (0)

#define GQ_TRY(expr)                 \
  do {                               \
    int _s = (expr);                 \
    if (_s != GQ_OK) return _s;      \
  } while (0)

#define GQ_REQUIRE(cond, ...)                                  \
  do {                                                         \
    if (!(cond)) return ::gq::fail(GQ_EINVAL, __VA_ARGS__);    \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Nanosecond clock for bounded spin waits.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Default upper bound for any device-side wait (a wait that outlives it
// records GQ_DEVERR_TIMEOUT in the kernel's status word and gives up).  Each
// translation unit with bounded waits keeps the bound in a __device__
// variable that gq_set_wait_limit_ns changes (tests shorten it to make a
// wait expire quickly).
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Device status word values written by kernels.
constexpr int GQ_DEVERR_NONE = 0;
constexpr int GQ_DEVERR_TIMEOUT = 1;
constexpr int GQ_DEVERR_NOTPD = 2;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Number of SMs of the current device (cached per device).
int sm_count();
// Grid size for persistent kernels: sm_count(), or less when this host thread
// set a budget with gq_set_cta_budget.
int cta_budget();
// Whether the bf16 statistics kernels run on CTA pairs; set with gq_set_pair_kernels.
bool pair_kernels();

}  // namespace gq
