// mlstm_recurrent.cu — step-by-step mLSTM recurrence on CUDA cores (sm_100a).
//
// The exact recurrence of tfla_forward_pytorch
// (hybrid_xmamba/kernels/tfla/tfla_interface.py:84-139):
//     C = f*C + i*k v^T,  n = f*n + i*k,  h = q C / max(q.n, 1)
// with per-head or per-key-channel gates (mlstm_block.py:117-129), fp32
// state, any dqk/dv, bf16 or fp32 I/O.  It serves fp32 I/O (exact-tolerance
// parity), per-channel gates and shapes the tensor-core chunkwise kernel does
// not cover.
//
// Stabilized state: every key row j carries its own log-scale m[j]
// (C[j,:] = exp(m[j]) Cs[j,:], n[j] = exp(m[j]) ns[j]) updated as
//     m' = max(m + log f, log i),  Cs = e^(m+log f-m') Cs + e^(log i-m') k v^T.
// The readout uses M = max_j m'[j]:  h = sum_j q_j e^(m'_j-M) Cs_j /
// max(sum_j q_j e^(m'_j-M) ns_j, e^(-M)) — algebraically the reference.
//
// Grid: (dv / kE column tiles, batch*heads); block 256 threads = 8 row
// groups x 32 columns; each thread keeps its C column slice in registers.
#include "capi_internal.h"
#include "common.cuh"
#include "mlstm.h"

namespace hxm {
namespace mlstm {

constexpr int kE = 32;       // value columns per CTA
constexpr int kRG = 8;       // row groups
constexpr int kThreads = kE * kRG;

// only: NULL (every (b, h)) or a device int per (b, h); then only the pairs
// whose entry equals `want` run (the rest of the grid returns at once).
template <typename T, int RPT>  // RPT = rows per thread = ceil(dqk / kRG)
__global__ void __launch_bounds__(kThreads) mlstm_recurrent_kernel(const Params p, const int* __restrict__ only,
                                                                   int want) {
  if (only && only[blockIdx.y] != want) return;  // uniform over the CTA
  extern __shared__ __align__(16) float sm[];
  const int dqk = p.dqk;
  float* q_s = sm;              // [dqk]  q~ = q * e^(m'-M)
  float* k_s = q_s + dqk;       // [dqk]  raw k
  float* a_s = k_s + dqk;       // [dqk]  decay coefficient of row j
  float* bk_s = a_s + dqk;      // [dqk]  e^(log i - m') k_j
  float* v_s = bk_s + dqk;      // [kE]
  float* part = v_s + kE;       // [kRG][kE] partial numerators
  float* red = part + kRG * kE; // [2*8] block reductions

  const int tid = threadIdx.x;
  const int e = tid % kE;       // column within tile
  const int rg = tid / kE;      // row group
  const int bh = blockIdx.y;
  const int b = bh / p.heads, hh = bh % p.heads;
  const int e0 = blockIdx.x * kE;
  const int col = e0 + e;
  const bool cvalid = col < p.dv;

  const T* qg = static_cast<const T*>(p.q) + b * p.sq[0] + hh * p.sq[1];
  const T* kg = static_cast<const T*>(p.k) + b * p.sk[0] + hh * p.sk[1];
  const T* vg = static_cast<const T*>(p.v) + b * p.sv[0] + hh * p.sv[1];
  T* hg = static_cast<T*>(p.h) + b * p.sh[0] + hh * p.sh[1];
  const float* lig = p.log_i + b * p.si[0] + hh * p.si[1];
  const float* lfg = p.log_f + b * p.sf[0] + hh * p.sf[1];

  // state: rows j = rg + kRG*r of column `col`
  float C[RPT];
  // per-row scale / normalizer: rows j = tid + kThreads*r2 owned by this thread
  constexpr int kRows2 = (RPT * kRG + kThreads - 1) / kThreads;
  float m_row[kRows2], n_row[kRows2];
  const float m0 = p.m0 ? p.m0[bh] : 0.f;
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int j = rg + kRG * r;
    C[r] = (p.C0 && j < dqk && cvalid) ? p.C0[((int64_t)bh * dqk + j) * p.dv + col] : 0.f;
  }
#pragma unroll
  for (int r2 = 0; r2 < kRows2; ++r2) {
    const int j = tid + kThreads * r2;
    m_row[r2] = m0;
    n_row[r2] = (p.n0 && j < dqk) ? p.n0[(int64_t)bh * dqk + j] : 0.f;
  }

  for (int t = 0; t < p.seqlen; ++t) {
    // 1. per-row gate coefficients and the new scales
    float mloc = -INFINITY;
#pragma unroll
    for (int r2 = 0; r2 < kRows2; ++r2) {
      const int j = tid + kThreads * r2;
      if (j < dqk) {
        const float li = lig[(int64_t)t * p.ti + (p.gate_mode ? j : 0)];
        const float lf = lfg[(int64_t)t * p.tf + (p.gate_mode ? j : 0)];
        const float kj = to_f32<T>(kg[(int64_t)t * p.tk + j]);
        const float mn = fmaxf(m_row[r2] + lf, li);
        const float a = __expf(m_row[r2] + lf - mn);
        const float bk = __expf(li - mn) * kj;
        a_s[j] = a;
        bk_s[j] = bk;
        n_row[r2] = a * n_row[r2] + bk;
        m_row[r2] = mn;
        mloc = fmaxf(mloc, mn);
      }
    }
    if (tid < kE) v_s[tid] = (e0 + tid < p.dv) ? to_f32<T>(vg[(int64_t)t * p.tv + e0 + tid]) : 0.f;
    // block max of m'
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if ((tid & 31) == 0) red[tid >> 5] = mloc;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) M = fmaxf(M, red[w]);
    // 2. q~ and the denominator
    float dloc = 0.f;
#pragma unroll
    for (int r2 = 0; r2 < kRows2; ++r2) {
      const int j = tid + kThreads * r2;
      if (j < dqk) {
        const float qt = to_f32<T>(qg[(int64_t)t * p.tq + j]) * __expf(m_row[r2] - M);
        q_s[j] = qt;
        dloc = fmaf(qt, n_row[r2], dloc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dloc += __shfl_xor_sync(0xffffffffu, dloc, o);
    __syncthreads();  // red[] reads of M done; q_s/a_s/bk_s/v_s visible
    if ((tid & 31) == 0) red[8 + (tid >> 5)] = dloc;
    // 3. column update and partial numerator
    const float vv = v_s[e];
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const int j = rg + kRG * r;
      if (j < dqk) {
        C[r] = fmaf(a_s[j], C[r], bk_s[j] * vv);
        acc = fmaf(q_s[j], C[r], acc);
      }
    }
    part[rg * kE + e] = acc;
    __syncthreads();
    if (tid < kE) {
      float num = 0.f;
#pragma unroll
      for (int g = 0; g < kRG; ++g) num += part[g * kE + tid];
      float den = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) den += red[8 + w];
      const float hv = num / fmaxf(den, __expf(-M));
      if (e0 + tid < p.dv) hg[(int64_t)t * p.th + e0 + tid] = from_f32<T>(hv);
    }
    __syncthreads();
  }

  // final state in the per-head scale M_T = max_j m[j] (written by column-tile 0 for n, m)
  float mloc = -INFINITY;
#pragma unroll
  for (int r2 = 0; r2 < kRows2; ++r2)
    if (tid + kThreads * r2 < dqk) mloc = fmaxf(mloc, m_row[r2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
  if ((tid & 31) == 0) red[tid >> 5] = mloc;
  __syncthreads();
  float MT = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) MT = fmaxf(MT, red[w]);
  // publish per-row rescale factors e^(m_j - M_T)
#pragma unroll
  for (int r2 = 0; r2 < kRows2; ++r2) {
    const int j = tid + kThreads * r2;
    if (j < dqk) {
      const float sc = __expf(m_row[r2] - MT);
      a_s[j] = sc;
      if (blockIdx.x == 0 && p.nT) p.nT[(int64_t)bh * dqk + j] = n_row[r2] * sc;
    }
  }
  if (blockIdx.x == 0 && tid == 0 && p.mT) p.mT[bh] = MT;
  __syncthreads();
  if (p.CT && cvalid) {
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      const int j = rg + kRG * r;
      if (j < dqk) p.CT[((int64_t)bh * dqk + j) * p.dv + col] = C[r] * a_s[j];
    }
  }
}

template <typename T, int RPT>
static hxm_status launch_rpt(const Params& p, cudaStream_t st, const int* only, int want) {
  const size_t smem = sizeof(float) * (4 * (size_t)p.dqk + kE + kRG * kE + 16);
  auto kern = mlstm_recurrent_kernel<T, RPT>;
  if (smem > 48 * 1024) HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dv + kE - 1) / kE, p.batch * p.heads);
  kern<<<grid, kThreads, smem, st>>>(p, only, want);
  return check_launch("hxm_mlstm_chunkwise_fwd (recurrent)");
}

template <typename T>
static hxm_status launch_t(const Params& p, cudaStream_t st, const int* only, int want) {
  const int rpt = (p.dqk + kRG - 1) / kRG;
  if (rpt <= 8) return launch_rpt<T, 8>(p, st, only, want);
  if (rpt <= 16) return launch_rpt<T, 16>(p, st, only, want);
  if (rpt <= 32) return launch_rpt<T, 32>(p, st, only, want);
  if (rpt <= 64) return launch_rpt<T, 64>(p, st, only, want);
  set_error("hxm_mlstm_chunkwise_fwd: dqk=%d > 512 unsupported by the recurrent kernel", p.dqk);
  return HXM_EUNSUPPORTED;
}

hxm_status launch_recurrent(const Params& p, cudaStream_t st, const int* only, int want) {
  if (p.io_dtype == HXM_F32) return launch_t<float>(p, st, only, want);
  return launch_t<__nv_bfloat16>(p, st, only, want);
}

}  // namespace mlstm
}  // namespace hxm
