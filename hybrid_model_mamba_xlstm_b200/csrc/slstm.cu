// slstm.cu — sLSTM recurrence: C ABI, and the general one-CTA-per-head kernel.
//
// Replaces the inline loop of sLSTMBlock.forward (hybrid_xmamba/layers/
// slstm_block.py:91-127):  i = exp (or sigmoid), f = sigmoid, o = sigmoid,
// c~ = tanh (:94-102); c = f*c + i*c~ (:119); h = o * tanh(RMSNorm_hd(c))
// (:122-125, normalization.py:32-34), plus the optional block-diagonal
// recurrent term R[head]^T h_{t-1} (absent in the reference).
//
// Exponential input gates are stabilized per channel:
//   m' = max(m + log f, log i),  cs = e^(m + log f - m') cs + e^(log i - m') c~,
// true cell c = e^m cs; RMSNorm uses M = max_j m_j:
//   c_j / rms(c) = e^(m_j - M) cs_j / sqrt(mean_j(e^(2(m_j-M)) cs_j^2) + eps e^(-2M)).
// With sigmoid input gates m stays 0 and this is the plain recurrence.
#include "capi_internal.h"
#include "common.cuh"
#include "slstm.h"

namespace hxm {
namespace slstm {

HXM_DEV float log_sigmoid(float x) { return fminf(x, 0.f) - log1pf(__expf(-fabsf(x))); }

// One CTA per (b, head), thread j owns channel j (hd <= 1024); the block is
// rounded up to whole warps and the extra lanes are neutral in the reductions.
template <typename T>
__global__ void slstm_simple_kernel(const Params p) {
  extern __shared__ float sm[];
  const int hd = p.hd;
  float* hprev = sm;           // [hd]
  float* red = sm + hd;        // [64]
  const int j = threadIdx.x;
  const bool act = j < hd;
  const int b = blockIdx.x / p.heads, hh = blockIdx.x % p.heads;
  const int nw = blockDim.x / 32;
  const T* g = static_cast<const T*>(p.gates);
  T* out = static_cast<T*>(p.h_out);
  const int64_t sstate = ((int64_t)b * p.heads + hh) * hd + (act ? j : 0);
  float c = (act && p.c0) ? p.c0[sstate] : 0.f;  // stabilized cell, m = 0 initially
  float m = 0.f;
  float h = (act && p.h0) ? p.h0[sstate] : 0.f;
  if (act) hprev[j] = h;
  const float wj = act ? p.w[j] : 0.f;
  const __nv_bfloat16* R = p.R ? p.R + (int64_t)hh * hd * 4 * hd : nullptr;
  __syncthreads();
  for (int t = 0; t < p.seqlen; ++t) {
    const T* gt = g + (((int64_t)b * p.seqlen + t) * p.heads + hh) * 4 * hd;
    float pre[4] = {0.f, 0.f, 0.f, 0.f};
    if (act) {
#pragma unroll
      for (int q = 0; q < 4; ++q) pre[q] = to_f32<T>(gt[q * hd + j]);
      if (R) {
        for (int k = 0; k < hd; ++k) {
          const float hk = hprev[k];
          const __nv_bfloat16* r = R + (int64_t)k * 4 * hd + j;
#pragma unroll
          for (int q = 0; q < 4; ++q) pre[q] = fmaf(hk, __bfloat162float(r[q * hd]), pre[q]);
        }
      }
    }
    const float lf = log_sigmoid(pre[1]);
    const float li = p.exp_gate ? pre[0] : log_sigmoid(pre[0]);
    const float mn = fmaxf(m + lf, li);
    c = __expf(m + lf - mn) * c + __expf(li - mn) * tanhf(pre[3]);
    m = mn;
    // block max of m, then sum of e^(2(m-M)) c^2
    float v = act ? m : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((j & 31) == 0) red[j >> 5] = v;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < nw; ++w) M = fmaxf(M, red[w]);
    const float sc = __expf(m - M);
    float s2 = act ? (sc * c) * (sc * c) : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    __syncthreads();
    if ((j & 31) == 0) red[32 + (j >> 5)] = s2;
    __syncthreads();
    float S = 0.f;
    for (int w = 0; w < nw; ++w) S += red[32 + w];
    const float rinv = rsqrtf(S / hd + p.eps * __expf(-2.f * M));
    const float og = 1.f / (1.f + __expf(-pre[2]));
    h = og * tanhf(wj * sc * c * rinv);
    if (act) {
      out[(((int64_t)b * p.seqlen + t) * p.heads + hh) * hd + j] = from_f32<T>(h);
      hprev[j] = h;
    }
    __syncthreads();
  }
  if (act && p.hT) p.hT[sstate] = h;
  if (act && p.cT) p.cT[sstate] = __expf(m) * c;
}

hxm_status launch_simple(const Params& p, cudaStream_t st) {
  const size_t smem = sizeof(float) * (p.hd + 64);
  dim3 grid(p.batch * p.heads);
  const int threads = (p.hd + 31) / 32 * 32;
  if (p.io_dtype == HXM_F32) slstm_simple_kernel<float><<<grid, threads, smem, st>>>(p);
  else slstm_simple_kernel<__nv_bfloat16><<<grid, threads, smem, st>>>(p);
  return check_launch("hxm_slstm_scan_fwd (simple)");
}

}  // namespace slstm
}  // namespace hxm

extern "C" hxm_status hxm_slstm_scan_fwd(const hxm_slstm_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_slstm_scan_fwd: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_slstm_args), "hxm_slstm_scan_fwd: struct_size %zu != %zu", a->struct_size,
              sizeof(hxm_slstm_args));
  HXM_REQUIRE(a->batch >= 0 && a->seqlen >= 0 && a->heads >= 0 && a->head_dim >= 1,
              "hxm_slstm_scan_fwd: bad dims B=%d L=%d H=%d hd=%d", a->batch, a->seqlen, a->heads, a->head_dim);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "hxm_slstm_scan_fwd: io_dtype must be f32 or bf16");
  HXM_REQUIRE_SUPPORTED(a->head_dim <= 1024, "hxm_slstm_scan_fwd: head_dim %d > 1024 unsupported", a->head_dim);
  HXM_REQUIRE(a->eps >= 0.f, "hxm_slstm_scan_fwd: eps must be >= 0");
  if (a->batch == 0 || a->heads == 0) return HXM_OK;
  HXM_REQUIRE(a->norm_weight != nullptr, "hxm_slstm_scan_fwd: norm_weight is NULL");
  HXM_REQUIRE(a->seqlen == 0 || (a->gates_pre && a->h_out), "hxm_slstm_scan_fwd: NULL tensor pointer");
  slstm::Params p{};
  p.batch = a->batch; p.seqlen = a->seqlen; p.heads = a->heads; p.hd = a->head_dim; p.io_dtype = a->io_dtype;
  p.gates = a->gates_pre; p.R = static_cast<const __nv_bfloat16*>(a->R); p.w = a->norm_weight; p.eps = a->eps;
  p.exp_gate = a->exponential_gate; p.h_out = a->h_out; p.h0 = a->h0; p.c0 = a->c0; p.hT = a->hT; p.cT = a->cT;
  p.error_flag = a->error_flag;
  p.wait_limit = a->wait_limit_cycles != 0 ? a->wait_limit_cycles : 4000000000ll;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.R && (p.hd == 128 || p.hd == 256) && p.seqlen > 0) {
    hxm_status s = slstm::launch_cluster(p, st);
    if (s != HXM_EUNSUPPORTED) return s;
    clear_error();
  }
  return slstm::launch_simple(p, st);
}
