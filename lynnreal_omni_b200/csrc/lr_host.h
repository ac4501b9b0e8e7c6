// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local error message, and argument checks. Internal to the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/lr_w8a8.h"

namespace lr {

// Record a formatted error message for lr_last_error() and return `status`.
int set_error(int status, const char* fmt, ...);

inline bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// Map the result of a kernel launch to a status code.
int launch_status(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace lr

#define LR_REQUIRE(cond, ...)                                              \
  do {                                                                     \
    if (!(cond)) return ::lr::set_error(LR_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)
