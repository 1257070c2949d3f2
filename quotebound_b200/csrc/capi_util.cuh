// The C ABI's error convention (the reference's, src/constrain_capi.h:7-9): -1 and a NUL-terminated
// reason in err; nothing throws across the boundary.  Shared by the files that define entry points.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

namespace qbgdn {

inline int capi_fail(char* err, int errlen, const char* fmt, ...) {
  if (err && errlen > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
    err[errlen - 1] = '\0';
  }
  return -1;
}

inline int capi_cuda(cudaError_t e, const char* what, char* err, int errlen) {
  if (e == cudaSuccess) return 0;
  return capi_fail(err, errlen, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

inline bool capi_aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace qbgdn
