// common.cuh — small device helpers shared by the hxm kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hxm.h"

#define HXM_DEV __device__ __forceinline__

namespace hxm {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---- dtype conversion ------------------------------------------------------
template <typename T> HXM_DEV float to_f32(T v);
template <> HXM_DEV float to_f32<float>(float v) { return v; }
template <> HXM_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> HXM_DEV float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> HXM_DEV T from_f32(float v);
template <> HXM_DEV float from_f32<float>(float v) { return v; }
template <> HXM_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> HXM_DEV __half from_f32<__half>(float v) { return __float2half_rn(v); }

// two floats -> one 32-bit word of two 16-bit values (one packed convert)
template <typename T> HXM_DEV uint32_t pack2(float lo, float hi);
template <> HXM_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> HXM_DEV uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---- hardware transcendental instructions (MUFU) ---------------------------
HXM_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
HXM_DEV float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
HXM_DEV float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
HXM_DEV float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softplus with torch's threshold (x > 20 -> x).
//   ACC: log1pf(expf(x)) from the CUDA math library (few-ulp accurate).
//   fast: ln2 * lg2(1 + 2^(x*log2e)) on the MUFU pipe; absolute error of the
//         result is ~1e-7, i.e. relative error <= 1e-4 for the smallest
//         outputs of interest (x >= -7) — far below bf16 output rounding.
template <bool ACC> HXM_DEV float softplus(float x) {
  if (ACC) return x > 20.f ? x : log1pf(expf(x));
  float e = ex2_approx(x * kLog2e);
  float s = kLn2 * lg2_approx(1.f + e);
  return x > 20.f ? x : s;
}

// sigmoid:  ACC -> 1/(1+expf(-x));  fast -> 0.5 + 0.5*tanh(x/2) (one MUFU op).
template <bool ACC> HXM_DEV float sigmoid(float x) {
  if (ACC) return 1.f / (1.f + expf(-x));
  return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
}

template <bool ACC> HXM_DEV float exp_(float x) {
  if (ACC) return expf(x);
  return ex2_approx(x * kLog2e);
}

// ---- async copies ----------------------------------------------------------
HXM_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// 16-byte global->shared async copy reading `src_bytes` (0..16) bytes and
// zero-filling the rest of the 16-byte destination.
HXM_DEV void cp_async16(void* smem_dst, const void* gmem_src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
HXM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> HXM_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

}  // namespace hxm
