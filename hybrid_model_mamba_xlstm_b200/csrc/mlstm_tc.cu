// mlstm_tc.cu — tcgen05 chunkwise mLSTM kernel (placeholder until built).
#include "capi_internal.h"
#include "mlstm.h"

namespace hxm {
namespace mlstm {
size_t chunkwise_tc_workspace(const Params&) { return (size_t)-1; }
hxm_status launch_chunkwise_tc(const Params&, cudaStream_t) {
  set_error("hxm_mlstm_chunkwise_fwd: tensor-core kernel not built");
  return HXM_EUNSUPPORTED;
}
}  // namespace mlstm
}  // namespace hxm
