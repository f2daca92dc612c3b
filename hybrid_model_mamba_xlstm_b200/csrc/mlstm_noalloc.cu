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
//     (scratch = 2 * B*H*L*dqk * 2 bytes + 3 * B*H*ceil(L/128)*dqk * 4 bytes,
//     each rounded up to 256 bytes).
//   - The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call
//     before any stream capture on the device.
//   - All calls share the one array and each call fully rewrites the part it
//     reads (nothing in it has to start at zero); calls whose executions
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
  hxm::clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_mlstm_chunkwise_fwd_noalloc: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_mlstm_args), "hxm_mlstm_chunkwise_fwd_noalloc: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_mlstm_args));
  HXM_REQUIRE(a->batch >= 0 && a->heads >= 0 && a->seqlen >= 0 && a->dqk >= 1 && a->dv >= 1,
              "hxm_mlstm_chunkwise_fwd_noalloc: bad dims");
  HXM_REQUIRE(a->gate_mode == 0 || a->gate_mode == 1, "hxm_mlstm_chunkwise_fwd_noalloc: bad gate_mode %d",
              a->gate_mode);
  Params p{};
  p.batch = a->batch; p.heads = a->heads; p.seqlen = a->seqlen; p.dqk = a->dqk; p.dv = a->dv;
  p.chunk = a->chunk; p.gate_mode = a->gate_mode; p.io_dtype = a->io_dtype;
  p.q = a->q; p.k = a->k; p.v = a->v; p.log_i = a->log_i; p.log_f = a->log_f; p.h = a->h;
  for (int i = 0; i < 2; ++i) {
    p.sq[i] = a->q_stride[i]; p.sk[i] = a->k_stride[i]; p.sv[i] = a->v_stride[i];
    p.si[i] = a->i_stride[i]; p.sf[i] = a->f_stride[i]; p.sh[i] = a->h_stride[i];
  }
  p.C0 = a->C0; p.n0 = a->n0; p.m0 = a->m0; p.CT = a->CT; p.nT = a->nT; p.mT = a->mT;
  hxm::mlstm::set_time_strides(p, a);
  if (p.batch == 0 || p.heads == 0 || p.seqlen == 0) {
    hxm::set_error("hxm_mlstm_chunkwise_fwd_noalloc: empty problem (batch, heads and seqlen must be > 0)");
    return HXM_EBADARG;
  }
  HXM_REQUIRE_SUPPORTED(hxm::mlstm::stream_shape_ok(p),
                        "hxm_mlstm_chunkwise_fwd_noalloc: needs bf16, dqk in {128, 256, 512}, dv %% 32 == 0 and "
                        "16-byte aligned v / h");
  HXM_REQUIRE(p.q && p.k && p.v && p.log_i && p.log_f && p.h, "hxm_mlstm_chunkwise_fwd_noalloc: NULL tensor pointer");
  const size_t need = hxm::mlstm::stream_workspace(p);
  HXM_REQUIRE(need <= kScratchBytes,
              "hxm_mlstm_chunkwise_fwd_noalloc: needs %zu bytes of scratch, the fixed device array holds %zu "
              "(32 MiB); use hxm_mlstm_chunkwise_fwd with a workspace",
              need, kScratchBytes);
  void* scratch = nullptr;
  hxm_status s = scratch_for_current_device(&scratch);
  if (s != HXM_OK) return s;
  p.workspace = scratch;
  p.workspace_bytes = kScratchBytes;
  return hxm::mlstm::launch_stream(p, static_cast<cudaStream_t>(stream));
}
