// nk_common.cuh — error plumbing and small helpers shared by every libnk
// translation unit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/nk.h"

namespace nk {

// ---------------------------------------------------------------- host errors
// Each API call records its outcome in a thread-local nk_error_info, the C
// counterpart of the Rust error enums' payloads.
nk_error_info &tls_error();

inline nk_status ok() {
  tls_error().code = NK_OK;
  return NK_OK;
}

inline nk_status fail(nk_status code, const char *msg) {
  nk_error_info &e = tls_error();
  memset(&e, 0, sizeof(e));
  e.code = code;
  snprintf(e.message, sizeof(e.message), "%s", msg);
  return code;
}

inline nk_status fail_length(const char *argument, uint64_t expected, uint64_t actual) {
  nk_error_info &e = tls_error();
  memset(&e, 0, sizeof(e));
  e.code = NK_LENGTH_MISMATCH;
  snprintf(e.argument, sizeof(e.argument), "%s", argument);
  e.expected = expected;
  e.actual = actual;
  snprintf(e.message, sizeof(e.message), "%s length mismatch: expected %llu, got %llu", argument,
           (unsigned long long)expected, (unsigned long long)actual);
  return NK_LENGTH_MISMATCH;
}

inline nk_status fail_cuda(cudaError_t err, const char *where) {
  char buf[200];
  snprintf(buf, sizeof(buf), "%s: %s", where, cudaGetErrorString(err));
  return fail(NK_DEVICE_ERROR, buf);
}

#define NK_CUDA_TRY(expr)                                  \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::nk::fail_cuda(_e, #expr); \
  } while (0)

// After a launch: surface launch-configuration errors immediately.
inline nk_status check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, what);
  return ok();
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------- device-side errors
// A bounded wait that gives up, or a kernel that detects a contract violation
// on the device, records a code here instead of trapping; nk_device_status()
// reads and clears it.  Codes: NK_TIMEOUT, NK_DEVICE_ERROR.
// Defined in common.cu; other units get its device address from device_error_ptr().
int *device_error_ptr();  // current device's error word (device address)

// Library scratch of the calling (device, stream) pair, grown on demand and
// never shrunk (nk_scratch_release frees it): split-K partial sums, reduction
// flags and staging buffers of the API calls that take no workspace argument.
nk_status scratch(size_t bytes, void **ptr, cudaStream_t stream);
nk_status release_scratch(cudaStream_t stream);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Overflow-checked products (the reference's checked_mul on usize).
inline bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
  return !__builtin_mul_overflow(a, b, out);
}

int num_sms();

}  // namespace nk

// ------------------------------------------------------------- device helpers
__device__ __forceinline__ float nk_relu2(float x) {
  float r = fmaxf(x, 0.0f);  // fmaxf(NaN, 0) = 0, as f32::max
  return r * r;
}

__device__ __forceinline__ uint64_t nk_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Two seconds: far beyond any legitimate wait inside one libnk kernel.
#define NK_WAIT_LIMIT_NS 2000000000ull
