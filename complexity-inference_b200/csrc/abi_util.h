// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local last-error message and argument checks.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/muk.h"

namespace muk {

void set_last_error(const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Returns MUK_ERR_CUDA (with the message) if the last launch failed.
int check_launch(const char* what);

}  // namespace muk

#define MUK_REQUIRE(cond, ...)            \
  do {                                    \
    if (!(cond)) {                        \
      ::muk::set_last_error(__VA_ARGS__); \
      return MUK_ERR_INVALID_ARG;         \
    }                                     \
  } while (0)

#define MUK_ALIGNED16(p) ((reinterpret_cast<uintptr_t>(p) & 15u) == 0)
