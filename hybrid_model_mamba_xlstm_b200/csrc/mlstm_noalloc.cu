// mlstm_noalloc.cu — hxm_mlstm_chunkwise_fwd_noalloc: the key-streaming
// tcgen05 mLSTM forward (per-channel gates or dqk up to 512) without any
// device allocation and without a caller-provided workspace.
//
// Some callers cannot allocate device memory when they run this op: plugin
// hosts whose execute/enqueue callbacks forbid cudaMalloc (it can block on or
// synchronize the device), and programs that reserve all device memory for
// their own pool up front and hand kernels only the tensors they own.  The
// streaming kernel needs scratch (the prescaled q / k copies and per-chunk
// decay vectors); this entry point takes it from a fixed-size array that
// the library itself places in device memory, so the caller only passes
// inputs and outputs.
//
// Contract
//   - Scratch: one file-scope device array of kScratchBytes = 32 MiB.  Every
//     GPU that loads this library holds those 32 MiB until the process exits.
//   - Requests whose scratch exceeds 32 MiB are rejected with HXM_EBADARG
//     (scratch = 2 * B*H*L*dqk * 2 bytes + 3 * B*H*ceil(L/64)*dqk * 4 bytes + B*H*L * 4 bytes
//     + B*H * 4 bytes, each rounded up to 256 bytes).
//   - The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current) and keeps it for the
//     life of the process; make that first call before any stream capture on
//     the device.  Resetting the device (cudaDeviceReset) after it is not
//     supported: the kept address would be stale.
//   - All calls share the one array.  Each call clears the part that must
//     start at zero (the per-(b, h) range flags, by cudaMemsetAsync) and
//     fully rewrites the rest before reading it; calls whose executions
//     overlap on the GPU (other streams, or other host threads) race on it.
//   - No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "capi_internal.h"
#include "mlstm.h"

namespace {

constexpr size_t kScratchBytes = 32u << 20;
static __device__ __align__(256) unsigned char g_mlstm_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_mlstm_scratch on the current device (resolved once per device).
hxm_status scratch_for_current_device(void** out) {
  int dev = 0;
  HXM_CUDA_TRY(cudaGetDevice(&dev));
  HXM_REQUIRE_SUPPORTED(dev >= 0 && dev < kMaxDevices, "hxm_mlstm_chunkwise_fwd_noalloc: device %d >= %d", dev,
                        kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_mlstm_scratch);
    if (e != cudaSuccess || !p) {
      hxm::set_error("hxm_mlstm_chunkwise_fwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return HXM_ECUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return HXM_OK;
}

}  // namespace

extern "C" hxm_status hxm_mlstm_chunkwise_fwd_noalloc(const hxm_mlstm_args* a, void* stream) {
  using hxm::mlstm::Params;
  static const char* who = "hxm_mlstm_chunkwise_fwd_noalloc";
  hxm::clear_error();
  Params p{};
  hxm_status s = hxm::mlstm::fill(a, p, who);  // the same argument checks as hxm_mlstm_chunkwise_fwd
  if (s != HXM_OK) return s;
  if (p.batch == 0 || p.heads == 0 || p.seqlen == 0) {
    hxm::set_error("%s: empty problem (batch, heads and seqlen must be > 0)", who);
    return HXM_EBADARG;
  }
  HXM_REQUIRE_SUPPORTED(hxm::mlstm::stream_shape_ok(p),
                        "%s: needs bf16, dqk in {128, 256, 512}, dv %% 32 == 0 and 16-byte aligned v / h", who);
  HXM_REQUIRE(p.q && p.k && p.v && p.log_i && p.log_f && p.h, "%s: NULL tensor pointer", who);
  const size_t need = hxm::mlstm::stream_workspace(p);
  HXM_REQUIRE(need <= kScratchBytes,
              "%s: needs %zu bytes of scratch, the fixed device array holds %zu (32 MiB); use "
              "hxm_mlstm_chunkwise_fwd with a workspace",
              who, need, kScratchBytes);
  void* scratch = nullptr;
  s = scratch_for_current_device(&scratch);
  if (s != HXM_OK) return s;
  p.workspace = scratch;  // args->workspace is ignored
  p.workspace_bytes = kScratchBytes;
  return hxm::mlstm::launch_stream(p, static_cast<cudaStream_t>(stream));
}
