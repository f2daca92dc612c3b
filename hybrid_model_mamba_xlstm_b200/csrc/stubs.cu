// stubs.cu — entry points declared in hxm.h whose kernels are not built yet.
// Each returns HXM_EUNSUPPORTED with a message; none touches the GPU.
#include "capi_internal.h"

extern "C" hxm_status hxm_slstm_scan_fwd(const hxm_slstm_args* a, void*) {
  HXM_REQUIRE(a && a->struct_size == sizeof(hxm_slstm_args), "hxm_slstm_scan_fwd: bad struct_size");
  hxm::set_error("hxm_slstm_scan_fwd: not built in this library version");
  return HXM_EUNSUPPORTED;
}
