// scan_inst_bf16_zoh.cu — instantiation of the selective-scan kernels for
// bf16 I/O with zoh discretization (own translation unit so the variants
// compile in parallel). 
#include "scan_kernel.cuh"

namespace hxm {
namespace scan {
hxm_status dispatch_bf16_zoh(const Params& p, cudaStream_t s, int num_sms) {
  return pick_ns<__nv_bfloat16, false, true>(p, s, num_sms);
}
}  // namespace scan
}  // namespace hxm
