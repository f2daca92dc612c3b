// capi.cu — library-level C ABI entry points and error plumbing.
#include "capi_internal.h"

namespace hxm {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

hxm_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return HXM_ECUDA;
  }
  return HXM_OK;
}

}  // namespace hxm

extern "C" int hxm_abi_version(void) { return HXM_ABI_VERSION; }

extern "C" const char* hxm_last_error_string(void) { return hxm::g_last_error.c_str(); }
