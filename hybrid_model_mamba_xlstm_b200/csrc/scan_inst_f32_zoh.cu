// scan_inst_f32_zoh.cu — instantiation of the selective-scan kernels
// for float I/O with zoh discretization (own translation unit so the
// variants compile in parallel).
#include "scan_kernel.cuh"

namespace hxm {
namespace scan {
hxm_status dispatch_f32_zoh(const Params& p, cudaStream_t s, int num_sms) {
  return pick_ns<float, true, true>(p, s, num_sms);
}
}  // namespace scan
}  // namespace hxm
