// capi_internal.h — shared plumbing of the C ABI implementation (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/hxm.h"

namespace hxm {

// Thread-local last-error message (returned by hxm_last_error_string()).
void set_error(const char* fmt, ...);
void clear_error();

// Returns HXM_ECUDA (with the message recorded) if the last launch failed.
hxm_status check_launch(const char* what);

inline size_t dtype_size(hxm_dtype t) { return t == HXM_F32 ? 4 : 2; }

}  // namespace hxm

#define HXM_REQUIRE(cond, ...)          \
  do {                                  \
    if (!(cond)) {                      \
      ::hxm::set_error(__VA_ARGS__);    \
      return HXM_EBADARG;               \
    }                                   \
  } while (0)

#define HXM_REQUIRE_SUPPORTED(cond, ...) \
  do {                                   \
    if (!(cond)) {                       \
      ::hxm::set_error(__VA_ARGS__);     \
      return HXM_EUNSUPPORTED;           \
    }                                    \
  } while (0)

#define HXM_CUDA_TRY(expr)                                                              \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess) {                                                            \
      ::hxm::set_error("%s failed: %s", #expr, cudaGetErrorString(e_));                 \
      return HXM_ECUDA;                                                                 \
    }                                                                                   \
  } while (0)
