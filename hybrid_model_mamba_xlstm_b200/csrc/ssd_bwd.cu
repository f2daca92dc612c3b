// ssd_bwd.cu — the per-head intra-chunk terms of the chunkwise SSD backward
// (sm_100a).
//
// The SSD recurrence (ngroups = 1: B, C shared by the heads; per-head scalar
// decay) has no reference kernel; its arithmetic is the Euler selective scan
// (hybrid_xmamba/kernels/selective_scan/scan_interface.py:132-150) with
// channel (head, p).  Within a chunk of c steps, with b the in-chunk prefix
// sum of the head's log decay dt A and CB = C B^T (shared by the heads):
//     S_h[t, s]  = CB[t, s] e^(b_t - b_s) dt_s          (s <= t, else 0)
// From G = dL/dS_h (a GEMM of dy and x per head) this kernel forms, one block
// per (batch, chunk) looping over the heads so the head sum stays on chip:
//     S_h                        (for dx = S_h^T dy)
//     M   = sum_h G e^(b_t - b_s) dt_s                 (dC += M B, dB += M^T C)
//     dti[s] = sum_t G CB e^(b_t - b_s)                 (dL/d dt_s, intra-chunk)
//     dbi[t] = rowsum(W)[t] - colsum(W)[t],  W = G * S_h without its diagonal
//                                                      (dL/d b_t, intra-chunk)
// The diagonal of W appears in both sums, so it is left out exactly.
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace ssd_bwd {

// C = chunk (32 or 64); 256 threads, thread = a fixed column s and C*C/256 rows
template <int C>
__global__ void __launch_bounds__(256) intra_kernel(const float* __restrict__ cb, const float* __restrict__ bcum,
                                                    const float* __restrict__ dt, const float* __restrict__ G,
                                                    int heads, float* __restrict__ S, float* __restrict__ M,
                                                    float* __restrict__ dti, float* __restrict__ dbi) {
  constexpr int kN = C * C / 256;  // elements per thread
  __shared__ float sb[C], sd[C], rowW[C], colW[C], colV[C];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t bk = blockIdx.x;  // batch * nchunks + chunk
  const int s = tid % C;          // this thread's column (256 % C == 0)
  float cbv[kN], macc[kN];
#pragma unroll
  for (int i = 0; i < kN; ++i) {
    cbv[i] = cb[bk * C * C + (int64_t)(256 * i + tid)];
    macc[i] = 0.f;
  }
#pragma unroll 1
  for (int h = 0; h < heads; ++h) {
    if (tid < C) {
      sb[tid] = bcum[(bk * C + tid) * heads + h];
      sd[tid] = dt[(bk * C + tid) * heads + h];
      rowW[tid] = colW[tid] = colV[tid] = 0.f;
    }
    __syncthreads();
    const float bs = sb[s], ds = sd[s];
    const int64_t tile = (bk * heads + h) * (int64_t)(C * C);
    float cw = 0.f, cv = 0.f;
#pragma unroll
    for (int i = 0; i < kN; ++i) {
      const int e = 256 * i + tid, t = e / C;
      const float g = G[tile + e];
      const float l = s <= t ? expf(sb[t] - bs) : 0.f;
      const float gl = g * l;
      S[tile + e] = cbv[i] * l * ds;
      macc[i] = fmaf(gl, ds, macc[i]);
      const float v = gl * cbv[i];
      cv += v;
      const float w = s == t ? 0.f : v * ds;
      cw += w;
      // row sum of W: the warp's 32 lanes share the row t
      float r = w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
      if (lane == 0) atomicAdd(&rowW[t], r);
    }
    atomicAdd(&colW[s], cw);
    atomicAdd(&colV[s], cv);
    __syncthreads();
    if (tid < C) {
      const int64_t o = (bk * heads + h) * C + tid;
      dti[o] = colV[tid];
      dbi[o] = rowW[tid] - colW[tid];
    }
    __syncthreads();  // the shared vectors are rewritten for the next head
  }
#pragma unroll
  for (int i = 0; i < kN; ++i) M[bk * C * C + (int64_t)(256 * i + tid)] = macc[i];
}

}  // namespace ssd_bwd
}  // namespace hxm

extern "C" hxm_status hxm_ssd_bwd_intra(const hxm_ssd_bwd_intra_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_ssd_bwd_intra: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_ssd_bwd_intra_args), "hxm_ssd_bwd_intra: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_ssd_bwd_intra_args));
  HXM_REQUIRE(a->batch >= 0 && a->nchunks >= 0 && a->heads >= 1, "hxm_ssd_bwd_intra: bad sizes batch=%d nchunks=%d heads=%d",
              a->batch, a->nchunks, a->heads);
  HXM_REQUIRE_SUPPORTED(a->chunk == 32 || a->chunk == 64, "hxm_ssd_bwd_intra: chunk %d (32 or 64 supported)",
                        a->chunk);
  const int64_t blocks = (int64_t)a->batch * a->nchunks;
  if (blocks == 0) return HXM_OK;
  HXM_REQUIRE(blocks < (int64_t)0x7fffffff, "hxm_ssd_bwd_intra: too many chunks (%lld)", (long long)blocks);
  HXM_REQUIRE(a->cb && a->bcum && a->dt && a->dS && a->S && a->M && a->ddt && a->db,
              "hxm_ssd_bwd_intra: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->chunk == 64)
    ssd_bwd::intra_kernel<64><<<(unsigned)blocks, 256, 0, st>>>(a->cb, a->bcum, a->dt, a->dS, a->heads, a->S, a->M,
                                                                 a->ddt, a->db);
  else
    ssd_bwd::intra_kernel<32><<<(unsigned)blocks, 256, 0, st>>>(a->cb, a->bcum, a->dt, a->dS, a->heads, a->S, a->M,
                                                                 a->ddt, a->db);
  return check_launch("hxm_ssd_bwd_intra");
}
