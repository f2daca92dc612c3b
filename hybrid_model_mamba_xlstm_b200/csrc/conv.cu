// conv.cu — causal depthwise conv1d (+ bias, + SiLU) for sm_100a.
//
// Replaces the Mamba pre-scan convolution (hybrid_xmamba/layers/
// mamba_block.py:101-104: rearrange, nn.Conv1d(groups=dim, padding=width-1),
// trim to seqlen, rearrange back, SiLU) with one pass over (batch, seqlen,
// channels) memory: HBM-bound, every input and output byte moves once.
//
// Unit channel stride, 16-byte aligned rows and whole 16-byte channel groups
// run the pipelined kernel (conv_pipe_kernel below: shared-memory tiles with
// three stages of 16-byte cp.async in flight).  With a ragged last channel
// group, the register-window kernel: a thread owns 16
// bytes of channels (8 bf16 / 4 fp32) and a run of kRun steps; it keeps the
// last width-1 inputs in registers, so each x row is read once with 16-byte
// loads (a warp reads 512 contiguous bytes per step) and each output row is
// written once with 16-byte stores.  The first width-1 inputs of a run come
// from the previous run's rows (or init_state / zeros before t = 0).
// Other strides run a one-thread-per-output element kernel.
#include <algorithm>

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

// Pipelined kernel (unit channel stride, 16-byte aligned rows, whole 16-byte channel groups):
// CTA = one batch row x a slab of kCG 16-byte channel groups x a run of `tiles` tiles of kR
// steps.  Tile i's rows t0 - (K-1) .. t0 + kR - 1 (the halo re-read from L2) are copied into
// shared memory with 16-byte cp.async while tiles i+1, i+2 are in flight (3 stages), so the
// loads of later tiles overlap this tile's arithmetic and stores; each thread then produces
// kRPT consecutive output rows of one channel group from a register window.  The
// register-window kernel above kept only its own 8-row load group in flight (2.0 TB/s at
// 8 x 2048 x 2048).
constexpr int kR = 32, kCG = 64, kRG = 4, kRPT = kR / kRG, kStages = 3, kPipeThreads = kCG * kRG;

template <typename T, int K>
__global__ void __launch_bounds__(kPipeThreads, 2) conv_pipe_kernel(const Params p, int tiles) {
  constexpr int V = 16 / sizeof(T);
  constexpr int H = K - 1;          // halo rows
  constexpr int kRows = kR + H;     // rows per stage
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint4* stages = reinterpret_cast<uint4*>(smem_raw);  // [kStages][kRows][kCG]
  const int tid = threadIdx.x, cg = tid % kCG, rg = tid / kCG;
  const int b = blockIdx.z;
  const int c0 = (blockIdx.y * kCG + cg) * V;  // this thread's first channel
  const bool cvalid = c0 < p.channels;         // channels is a multiple of V here
  const int tile0 = blockIdx.x * tiles;
  const int nt = min(tiles, (p.seqlen + kR - 1) / kR - tile0);
  if (nt <= 0) return;  // uniform over the CTA
  const T* xb = static_cast<const T*>(p.x) + b * p.sx[0];
  T* ob = static_cast<T*>(p.out) + b * p.so[0] + c0;

  auto issue = [&](int i) {
    uint4* dst = stages + (i % kStages) * kRows * kCG;
    const int t0 = (tile0 + i) * kR;
    for (int e = tid; e < kRows * kCG; e += kPipeThreads) {
      const int r = e / kCG, g = e % kCG;
      const int t = t0 - H + r, c = (blockIdx.y * kCG + g) * V;
      const bool ok = t >= 0 && t < p.seqlen && c < p.channels;  // others: zero-filled
      cp_async16(dst + r * kCG + g, ok ? xb + (int64_t)t * p.sx[1] + c : xb, ok ? 16 : 0);
    }
  };

  float wv[V][K], bv[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = cvalid ? c0 + j : 0;
#pragma unroll
    for (int k = 0; k < K; ++k) wv[j][k] = p.w[(int64_t)c * K + k];
    bv[j] = p.bias ? p.bias[c] : 0.f;
  }
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (i < nt) issue(i);
    cp_async_commit();  // one group per tile slot, empty past the run: the wait count stays uniform
  }
  for (int i = 0; i < nt; ++i) {
    if (i + kStages - 1 < nt) issue(i + kStages - 1);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // tile i's rows have landed (this thread's copies)
    __syncthreads();               // ... and every thread's
    const uint4* st = stages + (i % kStages) * kRows * kCG;
    const int t0 = (tile0 + i) * kR;
    if (H > 0 && t0 == 0 && p.init) {
      // rows before t = 0 come from the initial state (b, c, K-1), not zeros
      if (rg == 0 && cvalid) {
        uint4* hs = stages + (i % kStages) * kRows * kCG;
#pragma unroll
        for (int r = 0; r < H; ++r) {
          uint4 v;
          T* e = reinterpret_cast<T*>(&v);
#pragma unroll
          for (int j = 0; j < V; ++j)
            e[j] = static_cast<const T*>(p.init)[((int64_t)b * p.channels + c0 + j) * H + r];
          hs[r * kCG + cg] = v;
        }
      }
      __syncthreads();
    }
    if (cvalid) {
      const int j0 = rg * kRPT;  // tile rows j0 .. j0 + kRPT - 1; stage row of x[t0 + j - H + k] is j + k
      float win[K][V];
#pragma unroll
      for (int k = 0; k < H; ++k) {
        const uint4 v = st[(j0 + k) * kCG + cg];
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int j = 0; j < V; ++j) win[k][j] = to_f32<T>(e[j]);
      }
#pragma unroll
      for (int jj = 0; jj < kRPT; ++jj) {
        const int t = t0 + j0 + jj;
        const uint4 v = st[(j0 + jj + H) * kCG + cg];
        const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
        for (int j = 0; j < V; ++j) win[H][j] = to_f32<T>(e[j]);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          float acc = bv[j];
#pragma unroll
          for (int k = 0; k < K; ++k) acc = fmaf(wv[j][k], win[k][j], acc);
          oe[j] = from_f32<T>(act_fn<T>(acc, p.act));
        }
        if (t < p.seqlen) *reinterpret_cast<uint4*>(ob + (int64_t)t * p.so[1]) = o;
#pragma unroll
        for (int k = 0; k < H; ++k)
#pragma unroll
          for (int j = 0; j < V; ++j) win[k][j] = win[k + 1][j];
      }
    }
    __syncthreads();  // stage i % kStages is read before it is refilled
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
  if (fast && p.channels % V == 0) {
    // pipelined kernel: runs of `tiles` tiles per CTA
    static int num_sms[64] = {0};
    int dev = 0;
    HXM_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 64 && num_sms[dev] == 0)
      HXM_CUDA_TRY(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    const int sms = dev < 64 ? num_sms[dev] : 148;
    const int ntile = (p.seqlen + kR - 1) / kR, slabs = (p.channels / V + kCG - 1) / kCG;
    // runs per (slab, batch row) so that the whole grid is resident at two CTAs per SM
    const int64_t per = std::max<int64_t>(1, (int64_t)2 * sms / ((int64_t)slabs * p.batch));
    const int tiles = (int)std::max<int64_t>(1, (ntile + per - 1) / per);
    dim3 grid((ntile + tiles - 1) / tiles, slabs, p.batch);
    const int smem = kStages * (kR + p.width - 1) * kCG * 16;
    auto go = [&](auto kern) -> hxm_status {
      HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      kern<<<grid, kPipeThreads, smem, st>>>(p, tiles);
      return HXM_OK;
    };
    hxm_status s;
    switch (p.width) {
      case 1: s = go(conv_pipe_kernel<T, 1>); break;
      case 2: s = go(conv_pipe_kernel<T, 2>); break;
      case 3: s = go(conv_pipe_kernel<T, 3>); break;
      default: s = go(conv_pipe_kernel<T, 4>); break;
    }
    if (s != HXM_OK) return s;
  } else if (fast) {
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
