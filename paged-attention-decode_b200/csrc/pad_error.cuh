// pad_error.cuh -- the library's error reporting, shared by every translation
// unit of libpad_b200.so: a non-OK status always comes with a message that
// pad_last_error() returns on the calling thread.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "pad_b200.h"

namespace pad {

inline thread_local std::string g_last_error;

__attribute__((format(printf, 2, 3))) inline int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

inline int cuda_fail(cudaError_t e, const char* what) {
  return fail(PAD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace pad
