// conv.cu — causal depthwise conv1d (+ bias, + SiLU) for sm_100a.
//
// Replaces the Mamba pre-scan convolution (hybrid_xmamba/layers/
// mamba_block.py:101-104: rearrange, nn.Conv1d(groups=dim, padding=width-1),
// trim to seqlen, rearrange back, SiLU) with one pass over (batch, seqlen,
// channels) memory: HBM-bound, every input and output byte moves once.
//
// Fast kernel (unit channel stride, 16-byte aligned rows): a thread owns 16
// bytes of channels (8 bf16 / 4 fp32) and a run of kRun steps; it keeps the
// last width-1 inputs in registers, so each x row is read once with 16-byte
// loads (a warp reads 512 contiguous bytes per step) and each output row is
// written once with 16-byte stores.  The first width-1 inputs of a run come
// from the previous run's rows (or init_state / zeros before t = 0).
// Other strides run a one-thread-per-output element kernel.
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace conv {

struct Params {
  int batch, seqlen, channels, width;
  const void* x;
  int64_t sx[3];
  const float* w;
  const float* bias;
  void* out;
  int64_t so[3];
  const void* init;
  void* fin;
  int act;
};

constexpr int kRun = 32;  // steps per thread

template <typename T>
HXM_DEV float load_x(const Params& p, int b, int t, int c) {
  if (t >= 0) return to_f32<T>(static_cast<const T*>(p.x)[b * p.sx[0] + (int64_t)t * p.sx[1] + c * p.sx[2]]);
  if (!p.init) return 0.f;
  const int km1 = p.width - 1;
  return to_f32<T>(static_cast<const T*>(p.init)[((int64_t)b * p.channels + c) * km1 + (km1 + t)]);
}

// SiLU: the accurate sigmoid for fp32 I/O, the one-MUFU form below bf16 rounding
template <typename T>
HXM_DEV float act_fn(float v, int act) { return act ? v * sigmoid<sizeof(T) == 4>(v) : v; }

template <typename T, int K>
__global__ void __launch_bounds__(128) conv_fast_kernel(const Params p) {
  constexpr int V = 16 / sizeof(T);  // channels per thread
  const int cg = blockIdx.x * blockDim.x + threadIdx.x;
  const int c0 = cg * V;
  const int t0 = blockIdx.y * kRun;
  const int b = blockIdx.z;
  if (c0 >= p.channels) return;
  const int nv = min(V, p.channels - c0);

  float wv[V][K], bv[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = j < nv ? c0 + j : c0;
#pragma unroll
    for (int k = 0; k < K; ++k) wv[j][k] = p.w[(int64_t)c * K + k];
    bv[j] = p.bias ? p.bias[c] : 0.f;
  }
  // window[k] holds x[t - (K-1) + k] for the step being produced
  float win[K][V];
#pragma unroll
  for (int k = 0; k < K - 1; ++k)
#pragma unroll
    for (int j = 0; j < V; ++j) win[k][j] = j < nv ? load_x<T>(p, b, t0 - (K - 1) + k, c0 + j) : 0.f;

  const T* __restrict__ xb = static_cast<const T*>(p.x) + b * p.sx[0] + c0;
  T* __restrict__ ob = static_cast<T*>(p.out) + b * p.so[0] + c0;
  const int t_end = min(p.seqlen, t0 + kRun);
  // groups of 8 steps: the 8 row loads are issued together, then computed
  for (int tg = t0; tg < t_end; tg += 8) {
    uint4 raw[8];
    if (nv == V) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (tg + i < t_end) raw[i] = *reinterpret_cast<const uint4*>(xb + (int64_t)(tg + i) * p.sx[1]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (tg + i >= t_end) break;
      if (nv == V) {
        const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
        for (int j = 0; j < V; ++j) win[K - 1][j] = to_f32<T>(e[j]);
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) win[K - 1][j] = j < nv ? to_f32<T>(xb[(int64_t)(tg + i) * p.sx[1] + j]) : 0.f;
      }
      float ov[V];
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float acc = bv[j];
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(wv[j][k], win[k][j], acc);
        ov[j] = act_fn<T>(acc, p.act);
      }
      T* dst = ob + (int64_t)(tg + i) * p.so[1];
      if (nv == V) {
        uint4 o;
        T* e = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int j = 0; j < V; ++j) e[j] = from_f32<T>(ov[j]);
        *reinterpret_cast<uint4*>(dst) = o;
      } else {
        for (int j = 0; j < nv; ++j) dst[j] = from_f32<T>(ov[j]);
      }
#pragma unroll
      for (int k = 0; k < K - 1; ++k)
#pragma unroll
        for (int j = 0; j < V; ++j) win[k][j] = win[k + 1][j];
    }
  }
}

template <typename T>
__global__ void conv_generic_kernel(const Params p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n = (int64_t)p.batch * p.seqlen * p.channels;
  if (i >= n) return;
  const int c = (int)(i % p.channels);
  const int t = (int)((i / p.channels) % p.seqlen);
  const int b = (int)(i / ((int64_t)p.channels * p.seqlen));
  float acc = p.bias ? p.bias[c] : 0.f;
  for (int k = 0; k < p.width; ++k) acc = fmaf(p.w[(int64_t)c * p.width + k], load_x<T>(p, b, t - (p.width - 1) + k, c), acc);
  static_cast<T*>(p.out)[b * p.so[0] + (int64_t)t * p.so[1] + c * p.so[2]] = from_f32<T>(act_fn<T>(acc, p.act));
}

// final_state[b, c, j] = x[b, seqlen - (width-1) + j, c] (init_state before t = 0)
template <typename T>
__global__ void conv_state_kernel(const Params p) {
  const int km1 = p.width - 1;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)p.batch * p.channels * km1) return;
  const int j = (int)(i % km1);
  const int c = (int)((i / km1) % p.channels);
  const int b = (int)(i / ((int64_t)km1 * p.channels));
  static_cast<T*>(p.fin)[i] = from_f32<T>(load_x<T>(p, b, p.seqlen - km1 + j, c));
}

template <typename T>
hxm_status launch(const Params& p, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x), oa = reinterpret_cast<uintptr_t>(p.out);
  const bool fast = p.sx[2] == 1 && p.so[2] == 1 && xa % 16 == 0 && oa % 16 == 0 && p.sx[0] % V == 0 &&
                    p.sx[1] % V == 0 && p.so[0] % V == 0 && p.so[1] % V == 0;
  if (fast) {
    const int groups = (p.channels + V - 1) / V;
    dim3 grid((groups + 127) / 128, (p.seqlen + kRun - 1) / kRun, p.batch);
    switch (p.width) {
      case 1: conv_fast_kernel<T, 1><<<grid, 128, 0, st>>>(p); break;
      case 2: conv_fast_kernel<T, 2><<<grid, 128, 0, st>>>(p); break;
      case 3: conv_fast_kernel<T, 3><<<grid, 128, 0, st>>>(p); break;
      default: conv_fast_kernel<T, 4><<<grid, 128, 0, st>>>(p); break;
    }
  } else {
    const int64_t n = (int64_t)p.batch * p.seqlen * p.channels;
    conv_generic_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p);
  }
  hxm_status s = check_launch("hxm_causal_conv1d_fwd");
  if (s != HXM_OK || !p.fin || p.width == 1) return s;
  const int64_t ns = (int64_t)p.batch * p.channels * (p.width - 1);
  conv_state_kernel<T><<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(p);
  return check_launch("hxm_causal_conv1d_fwd (final state)");
}

}  // namespace conv
}  // namespace hxm

extern "C" hxm_status hxm_causal_conv1d_fwd(const hxm_conv1d_args* a, void* stream_) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_causal_conv1d_fwd: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_conv1d_args), "hxm_causal_conv1d_fwd: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_conv1d_args));
  HXM_REQUIRE(a->batch >= 0 && a->seqlen >= 0 && a->channels >= 0, "hxm_causal_conv1d_fwd: bad dims %d %d %d",
              a->batch, a->seqlen, a->channels);
  HXM_REQUIRE_SUPPORTED(a->width >= 1 && a->width <= 4, "hxm_causal_conv1d_fwd: width %d not in 1..4", a->width);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "hxm_causal_conv1d_fwd: io_dtype must be f32 or bf16");
  HXM_REQUIRE(a->activation == 0 || a->activation == 1, "hxm_causal_conv1d_fwd: bad activation %d", a->activation);
  HXM_REQUIRE((int64_t)a->batch <= 65535, "hxm_causal_conv1d_fwd: batch %d > 65535", a->batch);
  if (a->batch == 0 || a->channels == 0) return HXM_OK;
  HXM_REQUIRE(a->weight != nullptr, "hxm_causal_conv1d_fwd: weight is NULL");
  if (a->seqlen > 0) HXM_REQUIRE(a->x && a->out, "hxm_causal_conv1d_fwd: NULL x / out");
  HXM_REQUIRE(a->seqlen == 0 || a->x != a->out, "hxm_causal_conv1d_fwd: out must not alias x");
  conv::Params p{};
  p.batch = a->batch; p.seqlen = a->seqlen; p.channels = a->channels; p.width = a->width;
  p.x = a->x; p.w = a->weight; p.bias = a->bias; p.out = a->out; p.init = a->init_state; p.fin = a->final_state;
  p.act = a->activation;
  for (int i = 0; i < 3; ++i) { p.sx[i] = a->x_stride[i]; p.so[i] = a->out_stride[i]; }
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  if (a->seqlen == 0) {
    // nothing to convolve; the final state is the initial state
    if (p.fin && p.width > 1) {
      const size_t bytes = dtype_size(a->io_dtype) * (size_t)a->batch * a->channels * (a->width - 1);
      if (p.init) HXM_CUDA_TRY(cudaMemcpyAsync(p.fin, p.init, bytes, cudaMemcpyDeviceToDevice, st));
      else HXM_CUDA_TRY(cudaMemsetAsync(p.fin, 0, bytes, st));
    }
    return HXM_OK;
  }
  return a->io_dtype == HXM_F32 ? conv::launch<float>(p, st) : conv::launch<__nv_bfloat16>(p, st);
}
