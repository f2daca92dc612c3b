// ssd_bwd.cu — the per-head intra-chunk terms and the row assembly of the
// chunkwise SSD backward (sm_100a).
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
// A second kernel assembles, per (batch, chunk, step, head) row, dx from its
// intra-chunk part, the state part alpha * (B Y^T) and D * dy, and the
// row dot products the dt, log-decay and D gradients need.
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

// One warp per (batch, chunk, step t, head h) row of P values:
//   dx[b, kc*C + t, h, :] = dxi[h, t, :] + alpha[t, h] BY[t, h, :] + D[h] dy
//   xby[t, h] = x . BY,  dycz[t, h] = dy . CZ,  dyx[t, h] = dy . x
// xh, dyh, dxi head-major (batch*nch, H, C, P); BY, CZ (batch*nch, C, H, P);
// rows past seqlen write no dx.
__global__ void __launch_bounds__(256) rows_kernel(const float* __restrict__ xh, const float* __restrict__ dyh,
                                                   const float* __restrict__ dxi, const float* __restrict__ BY,
                                                   const float* __restrict__ CZ, const float* __restrict__ alpha,
                                                   const float* __restrict__ D, int nch, int C, int H, int P,
                                                   int seqlen, int64_t rows, float* __restrict__ dx,
                                                   float* __restrict__ xby, float* __restrict__ dycz,
                                                   float* __restrict__ dyx) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * 8ll + (threadIdx.x >> 5);  // ((bk * C + t) * H + h)
  if (row >= rows) return;
  const int h = (int)(row % H);
  const int64_t bt = row / H;
  const int t = (int)(bt % C);
  const int64_t bk = bt / C;
  const int kc = (int)(bk % nch);
  const int64_t bi = bk / nch;
  const int64_t hm = ((bk * H + h) * C + t) * (int64_t)P;  // head-major row
  const int64_t tm = row * (int64_t)P;                     // step-major row
  const float al = alpha[row];
  const float dd = D ? D[h] : 0.f;
  const int tg = kc * C + t;
  float* out = tg < seqlen ? dx + ((bi * seqlen + tg) * H + h) * (int64_t)P : nullptr;
  float a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int p = lane; p < P; p += 32) {
    const float xv = xh[hm + p], gv = dyh[hm + p], by = BY[tm + p];
    a1 = fmaf(xv, by, a1);
    a2 = fmaf(gv, CZ[tm + p], a2);
    a3 = fmaf(gv, xv, a3);
    if (out) out[p] = dxi[hm + p] + al * by + dd * gv;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    a2 += __shfl_xor_sync(0xffffffffu, a2, o);
    a3 += __shfl_xor_sync(0xffffffffu, a3, o);
  }
  if (lane == 0) {
    xby[row] = a1;
    dycz[row] = a2;
    if (dyx) dyx[row] = a3;
  }
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

extern "C" hxm_status hxm_ssd_bwd_rows(const hxm_ssd_bwd_rows_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_ssd_bwd_rows: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_ssd_bwd_rows_args), "hxm_ssd_bwd_rows: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_ssd_bwd_rows_args));
  HXM_REQUIRE(a->batch >= 0 && a->nchunks >= 0 && a->chunk >= 1 && a->heads >= 1 && a->headdim >= 1 &&
                  a->seqlen >= 0 && a->seqlen <= (int64_t)a->nchunks * a->chunk,
              "hxm_ssd_bwd_rows: bad sizes batch=%d nchunks=%d chunk=%d heads=%d headdim=%d seqlen=%d", a->batch,
              a->nchunks, a->chunk, a->heads, a->headdim, a->seqlen);
  const int64_t rows = (int64_t)a->batch * a->nchunks * a->chunk * a->heads;
  if (rows == 0) return HXM_OK;
  HXM_REQUIRE(a->xh && a->dyh && a->dxi && a->BY && a->CZ && a->alpha && a->dx && a->xby && a->dycz,
              "hxm_ssd_bwd_rows: NULL pointer");
  HXM_REQUIRE((rows + 7) / 8 < (int64_t)0x7fffffff, "hxm_ssd_bwd_rows: too many rows (%lld)", (long long)rows);
  ssd_bwd::rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a->xh, a->dyh, a->dxi, a->BY, a->CZ, a->alpha, a->D, a->nchunks, a->chunk, a->heads, a->headdim, a->seqlen,
      rows, a->dx, a->xby, a->dycz, a->dyx);
  return check_launch("hxm_ssd_bwd_rows");
}
