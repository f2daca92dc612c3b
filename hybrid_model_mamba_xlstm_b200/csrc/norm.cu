// norm.cu — RMSNorm over rows, optionally fused with the residual add before
// it (sm_100a).
//
// Replaces RMSNorm.forward (hybrid_xmamba/layers/normalization.py:32-34) and,
// fused, the residual add + next pre-norm of HybridBlock.forward
// (hybrid_xmamba/layers/hybrid_block.py:122-130).  HBM-bound: one read of x
// (and residual), one write of out (and the sum).
//
// Fast kernel (dim a multiple of 8, 16-byte aligned rows, dim <= 4096): one
// warp per row, each lane holding up to VPL 16-byte vectors of the row in
// registers, sum of squares by warp shuffles.  Otherwise one CTA per row
// with scalar loads.
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace norm {

struct Params {
  int64_t rows;
  int dim;
  const void* x;
  int64_t sx;
  const void* res;
  int64_t sr;
  void* sum;
  int64_t ss;
  const float* w;
  float eps;
  void* out;
  int64_t so;
};

template <typename T>
HXM_DEV void unpack(const uint4& raw, float (&v)[16 / sizeof(T)]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < (int)(16 / sizeof(T)); ++j) v[j] = to_f32<T>(e[j]);
}
template <typename T>
HXM_DEV uint4 pack(const float (&v)[16 / sizeof(T)]) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int j = 0; j < (int)(16 / sizeof(T)); ++j) e[j] = from_f32<T>(v[j]);
  return raw;
}

template <typename T, int VPL>
__global__ void __launch_bounds__(128) rmsnorm_warp_kernel(const Params p) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nvec = p.dim / V;
  const T* __restrict__ xr = static_cast<const T*>(p.x) + row * p.sx;
  const T* __restrict__ rr = p.res ? static_cast<const T*>(p.res) + row * p.sr : nullptr;
  float v[VPL][V];
  float ssq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = i * 32 + lane;
    if (c < nvec) {
      unpack<T>(*reinterpret_cast<const uint4*>(xr + c * V), v[i]);
      if (rr) {
        float r[V];
        unpack<T>(*reinterpret_cast<const uint4*>(rr + c * V), r);
#pragma unroll
        for (int j = 0; j < V; ++j) v[i][j] = to_f32<T>(from_f32<T>(v[i][j] + r[j]));  // the io-dtype sum
        if (p.sum) *reinterpret_cast<uint4*>(static_cast<T*>(p.sum) + row * p.ss + c * V) = pack<T>(v[i]);
      }
#pragma unroll
      for (int j = 0; j < V; ++j) ssq = fmaf(v[i][j], v[i][j], ssq);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
  const float rinv = rsqrtf(ssq / (float)p.dim + p.eps);
  T* orow = static_cast<T*>(p.out) + row * p.so;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = i * 32 + lane;
    if (c < nvec) {
      float o[V];
#pragma unroll
      for (int j = 0; j < V; ++j) o[j] = v[i][j] * rinv;
      if (p.w) {
        const float4* w4 = reinterpret_cast<const float4*>(p.w + c * V);
#pragma unroll
        for (int q = 0; q < V / 4; ++q) {
          const float4 wq = w4[q];
          o[4 * q] *= wq.x; o[4 * q + 1] *= wq.y; o[4 * q + 2] *= wq.z; o[4 * q + 3] *= wq.w;
        }
      }
      *reinterpret_cast<uint4*>(orow + c * V) = pack<T>(o);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_row_kernel(const Params p) {
  const int64_t row = blockIdx.x;
  const T* xr = static_cast<const T*>(p.x) + row * p.sx;
  const T* rr = p.res ? static_cast<const T*>(p.res) + row * p.sr : nullptr;
  float ssq = 0.f;
  for (int c = threadIdx.x; c < p.dim; c += blockDim.x) {
    float s = to_f32<T>(xr[c]);
    if (rr) s = to_f32<T>(from_f32<T>(s + to_f32<T>(rr[c])));
    ssq = fmaf(s, s, ssq);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ssq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rinv = rsqrtf(red[0] / (float)p.dim + p.eps);
  T* orow = static_cast<T*>(p.out) + row * p.so;
  T* srow = p.sum ? static_cast<T*>(p.sum) + row * p.ss : nullptr;
  for (int c = threadIdx.x; c < p.dim; c += blockDim.x) {
    float s = to_f32<T>(xr[c]);
    if (rr) {
      const T st = from_f32<T>(s + to_f32<T>(rr[c]));
      s = to_f32<T>(st);
      if (srow) srow[c] = st;
    }
    orow[c] = from_f32<T>((p.w ? p.w[c] : 1.f) * (s * rinv));
  }
}

template <typename T>
hxm_status launch(const Params& p, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  auto al = [&](const void* ptr, int64_t s) { return ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && s % V == 0); };
  const bool fast = p.dim % V == 0 && p.dim <= 512 * V && al(p.x, p.sx) && al(p.res, p.sr) && al(p.sum, p.ss) &&
                    al(p.out, p.so) && al(p.w, 0);
  if (fast) {
    const int vpl = (p.dim / V + 31) / 32;
    const unsigned grid = (unsigned)((p.rows + 3) / 4);
    if (vpl <= 1) rmsnorm_warp_kernel<T, 1><<<grid, 128, 0, st>>>(p);
    else if (vpl <= 2) rmsnorm_warp_kernel<T, 2><<<grid, 128, 0, st>>>(p);
    else if (vpl <= 4) rmsnorm_warp_kernel<T, 4><<<grid, 128, 0, st>>>(p);
    else if (vpl <= 8) rmsnorm_warp_kernel<T, 8><<<grid, 128, 0, st>>>(p);
    else rmsnorm_warp_kernel<T, 16><<<grid, 128, 0, st>>>(p);
  } else {
    rmsnorm_row_kernel<T><<<(unsigned)p.rows, 256, 0, st>>>(p);
  }
  return check_launch("hxm_rmsnorm_fwd");
}

}  // namespace norm
}  // namespace hxm

extern "C" hxm_status hxm_rmsnorm_fwd(const hxm_rmsnorm_args* a, void* stream_) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_rmsnorm_fwd: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_rmsnorm_args), "hxm_rmsnorm_fwd: struct_size %zu != %zu", a->struct_size,
              sizeof(hxm_rmsnorm_args));
  HXM_REQUIRE(a->rows >= 0 && a->dim >= 1, "hxm_rmsnorm_fwd: bad rows=%lld dim=%d", (long long)a->rows, a->dim);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "hxm_rmsnorm_fwd: io_dtype must be f32 or bf16");
  HXM_REQUIRE(a->rows <= 0x7fffffffLL, "hxm_rmsnorm_fwd: rows %lld too large", (long long)a->rows);
  if (a->rows == 0) return HXM_OK;
  HXM_REQUIRE(a->x && a->out, "hxm_rmsnorm_fwd: NULL x / out");
  HXM_REQUIRE(a->sum_out == nullptr || a->residual != nullptr, "hxm_rmsnorm_fwd: sum_out needs a residual");
  norm::Params p{};
  p.rows = a->rows; p.dim = a->dim;
  p.x = a->x; p.sx = a->x_row_stride;
  p.res = a->residual; p.sr = a->residual_row_stride;
  p.sum = a->sum_out; p.ss = a->sum_row_stride;
  p.w = a->weight; p.eps = a->eps;
  p.out = a->out; p.so = a->out_row_stride;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  return a->io_dtype == HXM_F32 ? norm::launch<float>(p, st) : norm::launch<__nv_bfloat16>(p, st);
}
