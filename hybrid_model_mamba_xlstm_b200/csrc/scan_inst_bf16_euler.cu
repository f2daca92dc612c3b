// scan_inst_bf16_euler.cu — instantiation of the selective-scan kernels
// for __nv_bfloat16 I/O with euler discretization (own translation unit so the
// variants compile in parallel).
#include "scan_kernel.cuh"

namespace hxm {
namespace scan {
hxm_status dispatch_bf16_euler(const Params& p, cudaStream_t s, int num_sms) {
  return pick_ns<__nv_bfloat16, false, false>(p, s, num_sms);
}
}  // namespace scan
}  // namespace hxm
