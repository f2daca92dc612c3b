// mlstm.h — shared parameter block of the mLSTM kernels (host + device).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hxm.h"

namespace hxm {
namespace mlstm {

constexpr int kChunk = 128;  // time chunk of the tensor-core kernels

struct Params {
  int batch, heads, seqlen, dqk, dv, chunk, gate_mode;
  hxm_dtype io_dtype;
  const void* q;
  int64_t sq[2];
  const void* k;
  int64_t sk[2];
  const void* v;
  int64_t sv[2];
  const float* log_i;
  int64_t si[2];
  const float* log_f;
  int64_t sf[2];
  void* h;
  int64_t sh[2];
  const float* C0;
  const float* n0;
  const float* m0;
  float* CT;
  float* nT;
  float* mT;
  void* workspace;
  size_t workspace_bytes;
  int64_t tq, tk, tv, th, ti, tf;  // time strides (elements)
  int* error_flag;                  // device int set to 1 when a bounded wait gave up, or NULL
  long long wait_limit;             // SM cycles per bounded device wait
};

// Time strides from the ABI struct (0 = dense).
inline void set_time_strides(Params& p, const hxm_mlstm_args* a) {
  const int64_t g = p.gate_mode == 1 ? p.dqk : 1;
  p.tq = a->q_tstride ? a->q_tstride : p.dqk;
  p.tk = a->k_tstride ? a->k_tstride : p.dqk;
  p.tv = a->v_tstride ? a->v_tstride : p.dv;
  p.th = a->h_tstride ? a->h_tstride : p.dv;
  p.ti = a->i_tstride ? a->i_tstride : g;
  p.tf = a->f_tstride ? a->f_tstride : g;
}

// Checks an hxm_mlstm_args and fills p (workspace included); `who` names the entry point in errors.
hxm_status fill(const hxm_mlstm_args* a, Params& p, const char* who);

// Exact step-by-step recurrence on CUDA cores (any gate mode / dtype / dims <= 512).
// only: NULL, or a device int per (b, h); then the pairs whose entry equals `want` run.
hxm_status launch_recurrent(const Params& p, cudaStream_t st, const int* only = nullptr, int want = 1);
// tcgen05 chunkwise kernel (bf16, per-head gates, dqk 128/256, stabilized); no workspace.
hxm_status launch_chunkwise_tc(const Params& p, cudaStream_t st);
size_t chunkwise_tc_workspace(const Params& p);  // (size_t)-1 when the shape is not covered
// Key-streaming tcgen05 kernel (bf16, per-head or per-channel gates, dqk 128/256/512) with a
// prescale pass into a caller-owned workspace of stream_workspace() bytes.  (b, h) pairs whose
// chunk scaling would leave the fp32 range (decided on the device by the prescale pass) are
// run by the exact recurrent kernel instead, in the same call.
bool stream_shape_ok(const Params& p);
size_t stream_workspace(const Params& p);
hxm_status launch_stream(const Params& p, cudaStream_t st);

}  // namespace mlstm
}  // namespace hxm
