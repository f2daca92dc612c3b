// slstm.h — shared parameter block of the sLSTM kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hxm.h"

namespace hxm {
namespace slstm {

struct Params {
  int batch, seqlen, heads, hd;
  hxm_dtype io_dtype;
  const void* gates;           // (b, t, heads, 4, hd)
  const __nv_bfloat16* R;      // (heads, hd, 4*hd) or null
  const float* w;              // (hd)
  float eps;
  int exp_gate;
  void* h_out;                 // (b, t, heads, hd)
  const float* h0;             // (b, heads, hd) true states, or null
  const float* c0;
  float* hT;
  float* cT;
  int* error_flag;
  long long wait_limit;        // cycles per bounded cross-CTA wait
};

hxm_status launch_simple(const Params& p, cudaStream_t st);
// Cluster kernel (hd 128 / 256, bf16 or fp32 gates); HXM_EUNSUPPORTED otherwise.
hxm_status launch_cluster(const Params& p, cudaStream_t st);

}  // namespace slstm
}  // namespace hxm
