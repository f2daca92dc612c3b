// scan_inst_bf16_euler.cu — instantiation of the selective-scan kernels for
// bf16 I/O with euler discretization (own translation unit so the variants
// compile in parallel).  The dominant time-major layout with dstate <= 16
// runs the packed-fp32x2 fast kernel; every other layout the generic one.
#include "scan_fast.cuh"

namespace hxm {
namespace scan {
hxm_status dispatch_bf16_euler(const Params& p, cudaStream_t s, int num_sms) {
  if (fast_ok(p, 2)) return pick_fast<__nv_bfloat16>(p, s, num_sms);
  return pick_ns<__nv_bfloat16, false, false>(p, s, num_sms);
}
}  // namespace scan
}  // namespace hxm
