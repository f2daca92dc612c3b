// mlstm.cu — C ABI of the mLSTM chunkwise forward (argument checks + dispatch).
//
// Replaces apply_tfla / TFLAFunction.forward / tfla_forward_pytorch
// (hybrid_xmamba/kernels/tfla/tfla_interface.py:18-49,84-139,142-163).
// bf16 I/O: per-head gates with dqk 128/256 run the fused tcgen05 chunkwise
// kernel; per-channel gates (mLSTMBlock) and dqk 512 run the key-streaming
// tcgen05 kernel (workspace: hxm_mlstm_workspace_size); fp32 I/O and other
// shapes run the exact CUDA-core recurrence.
#include "capi_internal.h"
#include "mlstm.h"

using hxm::mlstm::Params;

namespace hxm {
namespace mlstm {

hxm_status fill(const hxm_mlstm_args* a, Params& p, const char* who) {
  HXM_REQUIRE(a != nullptr, "%s: args is NULL", who);
  HXM_REQUIRE(a->struct_size == sizeof(hxm_mlstm_args), "%s: struct_size %zu != %zu", who, a->struct_size,
              sizeof(hxm_mlstm_args));
  HXM_REQUIRE(a->batch >= 0 && a->heads >= 0 && a->seqlen >= 0 && a->dqk >= 1 && a->dv >= 1,
              "%s: bad dims B=%d H=%d L=%d dqk=%d dv=%d", who, a->batch, a->heads, a->seqlen, a->dqk, a->dv);
  HXM_REQUIRE(a->gate_mode == 0 || a->gate_mode == 1, "%s: bad gate_mode %d", who, a->gate_mode);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "%s: io_dtype must be f32 or bf16", who);
  // The tensor-core kernels tile time in 128-step chunks (the chunkwise result does not depend on
  // the chunk length); other lengths are refused rather than silently replaced.
  HXM_REQUIRE_SUPPORTED(a->chunk == 0 || a->chunk == kChunk,
                        "%s: chunk %d unsupported (the kernels run %d-step chunks; pass 0 or %d)", who, a->chunk,
                        kChunk, kChunk, kChunk);
  HXM_REQUIRE_SUPPORTED(a->dqk <= 512 && a->dv <= 512, "%s: dqk, dv <= 512 supported", who);
  p.batch = a->batch; p.heads = a->heads; p.seqlen = a->seqlen; p.dqk = a->dqk; p.dv = a->dv;
  p.chunk = kChunk; p.gate_mode = a->gate_mode; p.io_dtype = a->io_dtype;
  p.q = a->q; p.k = a->k; p.v = a->v; p.log_i = a->log_i; p.log_f = a->log_f; p.h = a->h;
  for (int i = 0; i < 2; ++i) {
    p.sq[i] = a->q_stride[i]; p.sk[i] = a->k_stride[i]; p.sv[i] = a->v_stride[i];
    p.si[i] = a->i_stride[i]; p.sf[i] = a->f_stride[i]; p.sh[i] = a->h_stride[i];
  }
  p.C0 = a->C0; p.n0 = a->n0; p.m0 = a->m0; p.CT = a->CT; p.nT = a->nT; p.mT = a->mT;
  set_time_strides(p, a);
  p.workspace = a->workspace; p.workspace_bytes = a->workspace_bytes;
  p.error_flag = a->error_flag;
  p.wait_limit = a->wait_limit_cycles != 0 ? a->wait_limit_cycles : 4000000000ll;
  return HXM_OK;
}

}  // namespace mlstm
}  // namespace hxm

using hxm::mlstm::fill;

static bool use_tc(const Params& p) {
  return p.io_dtype == HXM_BF16 && p.gate_mode == 0 && hxm::mlstm::chunkwise_tc_workspace(p) != (size_t)-1;
}
static bool use_stream(const Params& p) { return !use_tc(p) && hxm::mlstm::stream_shape_ok(p); }

extern "C" size_t hxm_mlstm_workspace_size(const hxm_mlstm_args* a) {
  Params p{};
  if (fill(a, p, "hxm_mlstm_workspace_size") != HXM_OK) return 0;
  if (use_tc(p)) return hxm::mlstm::chunkwise_tc_workspace(p);
  return use_stream(p) ? hxm::mlstm::stream_workspace(p) : 0;
}

extern "C" hxm_status hxm_mlstm_chunkwise_fwd(const hxm_mlstm_args* a, void* stream) {
  hxm::clear_error();
  Params p{};
  hxm_status s = fill(a, p, "hxm_mlstm_chunkwise_fwd");
  if (s != HXM_OK) return s;
  if (p.batch == 0 || p.heads == 0) return HXM_OK;
  HXM_REQUIRE(p.seqlen == 0 || (p.q && p.k && p.v && p.log_i && p.log_f && p.h),
              "hxm_mlstm_chunkwise_fwd: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_tc(p)) return hxm::mlstm::launch_chunkwise_tc(p, st);
  if (use_stream(p)) return hxm::mlstm::launch_stream(p, st);
  return hxm::mlstm::launch_recurrent(p, st);
}
