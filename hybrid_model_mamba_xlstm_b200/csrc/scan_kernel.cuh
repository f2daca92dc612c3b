// scan.cu — fused Mamba selective scan for sm_100a (CUDA cores).
//
// Replaces selective_scan_pytorch / SelectiveScanFunction.forward
// (hybrid_xmamba/kernels/selective_scan/scan_interface.py:17-60,103-152) and
// selective_scan_fwd_kernel (scan_triton.py:31-192).  One thread owns one
// (batch, channel) recurrence with its dstate fp32 states in registers and
// walks the sequence tile by tile.  Per tile of T timesteps a CTA of CH
// channels (all of one batch row) stages u / delta / z with 16-byte cp.async
// (double buffered) and the shared B_t, C_t rows (converted to fp32) in
// shared memory, so every HBM byte is read once with 128-bit transactions and
// B, C are read once per CTA instead of once per channel.
//
// Fused per step: softplus(delta + bias), exp(delta*A) (as powers of one
// exp when A[d, n] = (n+1) * A[d, 0], checked on the device per warp), the
// Euler (reference) or ZOH update, the C.h + D*u readout and the z gate
// (y*z or y*silu(z)).  y overwrites u's staging slot and leaves with 16-byte
// stores.
#pragma once
#include "capi_internal.h"
#include "common.cuh"

#include <cmath>

namespace hxm {
namespace scan {


// Tensor I/O mode of u / delta / z / y:
//   kGeneric  element loads with arbitrary strides, staged time-major
//   kTimeMaj  unit time stride, 16B-aligned rows: async copy, [CH][T+pad]
//   kChanMaj  unit channel stride, 16B-aligned rows: async copy, [T][CH]
enum IoMode : int { kGeneric = 0, kTimeMaj = 1, kChanMaj = 2 };

struct Params {
  int batch, seqlen, dim, dstate;
  const void* u;
  int64_t su[3];
  const void* dt;
  int64_t sdt[3];
  const float* A;
  int64_t sA[2];
  const void* B;
  int64_t sB[3];
  const void* C;
  int64_t sC[3];
  const float* D;
  const void* z;
  int64_t sz[3];
  const float* bias;
  void* y;
  int64_t sy[3];
  const float* h0;
  float* hT;
  int z_mode, softplus;
  int mode_u, mode_dt, mode_z, mode_y;
  // time segments of the fast kernel (nseg = 1: one pass over the whole sequence).  Segment s
  // covers steps [s * seg_len, min((s + 1) * seg_len, seqlen)); seg_ws holds, per (batch,
  // channel) and segment s < nseg - 1, the state that segment reaches from zero (dstate <= 16
  // floats, padded to 16) and its sum of delta: 17 floats.
  float* seg_ws;
  int seg_len, nseg;
};

template <typename T, int CH, int kT>
struct Smem {
  static constexpr int kPad = 16 / sizeof(T);  // 16-byte row padding (bank spread)
  static constexpr int kTP = kT + kPad;        // time-major row pitch (elements)
  static constexpr int kSlot = (CH * kTP > kT * CH) ? CH * kTP : kT * CH;
};

// Element (ch, t) of a staging slot in its layout.
template <typename T, int CH, int kT>
HXM_DEV int slot_index(int mode, int ch, int t) {
  return mode == kChanMaj ? t * CH + ch : ch * Smem<T, CH, kT>::kTP + t;
}

// Issue the loads of one u/delta/z tile into a staging slot.  Async modes
// use cp.async (caller commits); the generic mode loads synchronously.
template <typename T, int CH, int kT>
HXM_DEV void load_io_tile(T* slot, int mode, const T* __restrict__ g, const int64_t* s, int b, int d0, int t0,
                          int tk, int dim) {
  const int tid = threadIdx.x;
  constexpr int kE = 16 / sizeof(T);  // elements per 16 bytes
  if (mode == kTimeMaj) {
    constexpr int kChunks = kT / kE;  // chunks per channel row
    for (int c = tid; c < CH * kChunks; c += CH) {
      const int ch = c / kChunks, part = c % kChunks;
      const int d = d0 + ch, t = part * kE;
      T* dst = slot + ch * Smem<T, CH, kT>::kTP + t;
      int valid = (d < dim) ? min(kE, tk - t) : 0;
      valid = max(valid, 0);
      const T* src = g + b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)(d < dim ? d : 0) * s[2];
      cp_async16(dst, valid > 0 ? src : g, valid * (int)sizeof(T));
    }
  } else if (mode == kChanMaj) {
    constexpr int kChunks = CH / kE;  // chunks per timestep row
    for (int c = tid; c < kT * kChunks; c += CH) {
      const int t = c / kChunks, part = c % kChunks;
      const int ch = part * kE, d = d0 + ch;
      T* dst = slot + t * CH + ch;
      int valid = (t < tk) ? min(kE, dim - d) : 0;
      valid = max(valid, 0);
      const T* src = g + b * s[0] + (int64_t)(t0 + (t < tk ? t : 0)) * s[1] + (int64_t)(valid > 0 ? d : 0) * s[2];
      cp_async16(dst, valid > 0 ? src : g, valid * (int)sizeof(T));
    }
  } else {
    // generic: walk with the unit-stride axis (if any) fastest for coalescing
    const bool tfast = s[1] == 1;
    for (int e = tid; e < CH * kT; e += CH) {
      const int ch = tfast ? e / kT : e % CH;
      const int t = tfast ? e % kT : e / CH;
      const int d = d0 + ch;
      T v = from_f32<T>(0.f);
      if (d < dim && t < tk) v = g[b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)d * s[2]];
      slot[ch * Smem<T, CH, kT>::kTP + t] = v;
    }
  }
}

// Store the y tile (held in u's staging slot, layout `smode`).
template <typename T, int CH, int kT>
HXM_DEV void store_y_tile(const T* slot, int smode, int ymode, T* __restrict__ g, const int64_t* s, int b, int d0,
                          int t0, int tk, int dim) {
  const int tid = threadIdx.x;
  constexpr int kE = 16 / sizeof(T);
  if (ymode == kTimeMaj && smode != kChanMaj) {
    constexpr int kChunks = kT / kE;
    for (int c = tid; c < CH * kChunks; c += CH) {
      const int ch = c / kChunks, t = (c % kChunks) * kE;
      const int d = d0 + ch;
      if (d >= dim || t >= tk) continue;
      const T* src = slot + ch * Smem<T, CH, kT>::kTP + t;
      T* dst = g + b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)d * s[2];
      if (t + kE <= tk) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      } else {
        for (int j = 0; j < tk - t; ++j) dst[j] = src[j];
      }
    }
  } else if (ymode == kChanMaj && smode == kChanMaj) {
    constexpr int kChunks = CH / kE;
    for (int c = tid; c < kT * kChunks; c += CH) {
      const int t = c / kChunks, ch = (c % kChunks) * kE;
      const int d = d0 + ch;
      if (t >= tk || d >= dim) continue;
      const T* src = slot + t * CH + ch;
      T* dst = g + b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)d * s[2];
      if (d + kE <= dim) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      } else {
        for (int j = 0; j < dim - d; ++j) dst[j] = src[j];
      }
    }
  } else {
    const bool tfast = s[1] == 1;
    for (int e = tid; e < CH * kT; e += CH) {
      const int ch = tfast ? e / kT : e % CH;
      const int t = tfast ? e % kT : e / CH;
      const int d = d0 + ch;
      if (d < dim && t < tk)
        g[b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)d * s[2]] = slot[slot_index<T, CH, kT>(smode, ch, t)];
    }
  }
}

// Read 8 consecutive timesteps (t0..t0+7) of channel `ch` from a slot.
template <typename T, int CH, int kT>
HXM_DEV void read8(const T* slot, int mode, int ch, int t0, float (&v)[8]) {
  if (mode != kChanMaj) {
    const T* p = slot + ch * Smem<T, CH, kT>::kTP + t0;
    if constexpr (sizeof(T) == 2) {
      uint4 w = *reinterpret_cast<const uint4*>(p);
      const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = to_f32<T>(e[j]);
    } else {
      float4 a = *reinterpret_cast<const float4*>(p);
      float4 c = *reinterpret_cast<const float4*>(p + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32<T>(slot[(t0 + j) * CH + ch]);
  }
}

template <typename T, int CH, int kT>
HXM_DEV void write8(T* slot, int mode, int ch, int t0, const float (&v)[8]) {
  if (mode != kChanMaj) {
    T* p = slot + ch * Smem<T, CH, kT>::kTP + t0;
    if constexpr (sizeof(T) == 2) {
      uint4 w;
      uint32_t* e = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int j = 0; j < 4; ++j) e[j] = pack2<T>(v[2 * j], v[2 * j + 1]);
      *reinterpret_cast<uint4*>(p) = w;
    } else {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) slot[(t0 + j) * CH + ch] = from_f32<T>(v[j]);
  }
}

// Per-thread register prefetch of one B/C tile (kT x NS each), converted to fp32.
template <typename T, int NS, int CH, int kT>
struct BCPrefetch {
  static constexpr int kElems = 2 * kT * NS;
  static constexpr int kPer = (kElems + CH - 1) / CH;
  float v[kPer];

  HXM_DEV void load(const Params& p, int b, int t0, int tk) {
    const T* Bg = static_cast<const T*>(p.B);
    const T* Cg = static_cast<const T*>(p.C);
    const int tid = threadIdx.x;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = tid + i * CH;
      float val = 0.f;
      if (e < kElems) {
        const int which = e / (kT * NS);  // 0 = B, 1 = C
        const int r = e % (kT * NS);
        const int64_t* s = which ? p.sC : p.sB;
        const T* g = which ? Cg : Bg;
        const bool tfast = s[1] == 1;
        const int t = tfast ? r % kT : r / NS;
        const int n = tfast ? r / kT : r % NS;
        if (t < tk && n < p.dstate) val = to_f32<T>(g[b * s[0] + (int64_t)(t0 + t) * s[1] + (int64_t)n * s[2]]);
      }
      v[i] = val;
    }
  }
  // smem layout: bc[t][0..NS) = B_t, bc[t][NS..2NS) = C_t
  HXM_DEV void store(float* bc, const Params& p) const {
    const int tid = threadIdx.x;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = tid + i * CH;
      if (e < kElems) {
        const int which = e / (kT * NS);
        const int r = e % (kT * NS);
        const int64_t* s = which ? p.sC : p.sB;
        const bool tfast = s[1] == 1;
        const int t = tfast ? r % kT : r / NS;
        const int n = tfast ? r / kT : r % NS;
        bc[t * 2 * NS + which * NS + n] = v[i];
      }
    }
  }
};

// One recurrence step for one channel.  Returns C.h (+ nothing else).
//   POW: exp(delta*A[n]) = r^(n+1), r = exp(delta*A[0]) (checked pattern).
template <bool ACC, bool ZOH, bool POW, int NS>
HXM_DEV float ssm_step(float dl, float u, const float* __restrict__ bc, float (&h)[NS], const float (&Al2)[NS],
                       const float (&Aval)[NS], const float (&invA)[NS]) {
  const float4* b4 = reinterpret_cast<const float4*>(bc);
  const float4* c4 = reinterpret_cast<const float4*>(bc + NS);
  float y0 = 0.f, y1 = 0.f;
  if (POW) {
    const float r = ex2_approx(dl * Al2[0]);
    const float du = dl * u;
    float pw = r;
#pragma unroll
    for (int q = 0; q < NS / 4; ++q) {
      const float4 bb = b4[q], cc = c4[q];
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
      const float cv[4] = {cc.x, cc.y, cc.z, cc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = 4 * q + j;
        h[n] = fmaf(pw, h[n], du * bv[j]);
        if (j & 1) y1 = fmaf(cv[j], h[n], y1); else y0 = fmaf(cv[j], h[n], y0);
        pw *= r;
      }
    }
  } else {
    const float du = dl * u;
#pragma unroll
    for (int q = 0; q < NS / 4; ++q) {
      const float4 bb = b4[q], cc = c4[q];
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
      const float cv[4] = {cc.x, cc.y, cc.z, cc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = 4 * q + j;
        const float dA = ACC ? expf(dl * Aval[n]) : ex2_approx(dl * Al2[n]);
        float bbar;
        if (ZOH) {
          const float x = dl * Aval[n];
          bbar = (fabsf(x) < 0.01f) ? du * bv[j] : (dA - 1.f) * invA[n] * bv[j] * u;
        } else {
          bbar = du * bv[j];
        }
        h[n] = fmaf(dA, h[n], bbar);
        if (j & 1) y1 = fmaf(cv[j], h[n], y1); else y0 = fmaf(cv[j], h[n], y0);
      }
    }
  }
  return y0 + y1;
}

// One staged tile of kT steps for one channel.  Branch-free step bodies:
// steps past the end of the sequence get delta = 0 (h unchanged, y unused).
template <typename T, int NS, int CH, int kT, bool ACC, bool ZOH, bool POW>
HXM_DEV void compute_tile(T* us, const T* ds, const T* zs, int mode_u, int mode_dt, int mode_z, bool has_z,
                          const float* __restrict__ bc, int tk, float (&h)[NS], const float (&Al2)[NS],
                          const float (&Aval)[NS], const float (&invA)[NS], float bias, float Dd, bool sp,
                          int z_mode, int tid) {
  const bool vec = mode_u != kChanMaj && mode_dt != kChanMaj && (!has_z || mode_z != kChanMaj);
  if (vec) {
#pragma unroll 1
    for (int tt = 0; tt < kT; tt += 8) {
      float uv[8], dv[8], zv[8], yv[8];
      read8<T, CH, kT>(us, kTimeMaj, tid, tt, uv);
      read8<T, CH, kT>(ds, kTimeMaj, tid, tt, dv);
      if (has_z) {
        read8<T, CH, kT>(zs, kTimeMaj, tid, tt, zv);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) zv[j] = 1.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float dl = dv[j] + bias;
        dl = sp ? softplus<ACC>(dl) : dl;
        dl = (tt + j < tk) ? dl : 0.f;
        float yy = ssm_step<ACC, ZOH, POW, NS>(dl, uv[j], bc + (tt + j) * 2 * NS, h, Al2, Aval, invA);
        yy = fmaf(Dd, uv[j], yy);
        const float g = (z_mode == 2) ? zv[j] * sigmoid<ACC>(zv[j]) : (z_mode == 1 ? zv[j] : 1.f);
        yv[j] = yy * g;
      }
      write8<T, CH, kT>(us, kTimeMaj, tid, tt, yv);
    }
  } else {
#pragma unroll 1
    for (int t = 0; t < tk; ++t) {
      const float u = to_f32<T>(us[slot_index<T, CH, kT>(mode_u, tid, t)]);
      float dl = to_f32<T>(ds[slot_index<T, CH, kT>(mode_dt, tid, t)]) + bias;
      dl = sp ? softplus<ACC>(dl) : dl;
      float yy = ssm_step<ACC, ZOH, POW, NS>(dl, u, bc + t * 2 * NS, h, Al2, Aval, invA);
      yy = fmaf(Dd, u, yy);
      if (has_z) {
        const float z = to_f32<T>(zs[slot_index<T, CH, kT>(mode_z, tid, t)]);
        yy *= (z_mode == 2) ? z * sigmoid<ACC>(z) : z;
      }
      us[slot_index<T, CH, kT>(mode_u, tid, t)] = from_f32<T>(yy);
    }
  }
}

template <typename T, int NS, int CH, int kT, bool ACC, bool ZOH>
__global__ void __launch_bounds__(CH) scan_fwd_kernel(const Params p) {
  using S = Smem<T, CH, kT>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* io = reinterpret_cast<T*>(smem_raw);                                   // [2][3][kSlot]
  float* bcs = reinterpret_cast<float*>(smem_raw + sizeof(T) * 2 * 3 * S::kSlot);  // [2][kT][2NS]

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * CH;
  const int d = d0 + tid;
  const bool dvalid = d < p.dim;
  const int dc = dvalid ? d : 0;

  // per-channel constants
  float Al2[NS], Aval[NS], invA[NS], h[NS];
  bool pattern = true;
  const float a0 = p.A[(int64_t)dc * p.sA[0]];
#pragma unroll
  for (int n = 0; n < NS; ++n) {
    const float a = n < p.dstate ? p.A[(int64_t)dc * p.sA[0] + (int64_t)n * p.sA[1]] : 0.f;
    Aval[n] = a;
    Al2[n] = a * kLog2e;
    invA[n] = (a != 0.f) ? 1.f / a : 0.f;
    if (n < p.dstate && a != a0 * (float)(n + 1)) pattern = false;
    h[n] = (p.h0 && dvalid && n < p.dstate) ? p.h0[((int64_t)b * p.dim + d) * p.dstate + n] : 0.f;
  }
  // exp(delta*A[n]) as powers of r = exp(delta*A[0]) — fast path only, decided per warp
  const bool use_pow = __all_sync(0xffffffffu, pattern);
  const float Dd = (p.D && dvalid) ? p.D[d] : 0.f;
  const float bias = (p.bias && dvalid) ? p.bias[d] : 0.f;

  const T* ug = static_cast<const T*>(p.u);
  const T* dtg = static_cast<const T*>(p.dt);
  const T* zg = static_cast<const T*>(p.z);
  T* yg = static_cast<T*>(p.y);
  const int ntiles = (p.seqlen + kT - 1) / kT;
  const int mode_z = p.z ? p.mode_z : kGeneric;

  auto slot = [&](int stage, int which) { return io + (stage * 3 + which) * S::kSlot; };
  auto issue = [&](int k) {
    const int st = k & 1, t0 = k * kT, tk = min(kT, p.seqlen - t0);
    load_io_tile<T, CH, kT>(slot(st, 0), p.mode_u, ug, p.su, b, d0, t0, tk, p.dim);
    load_io_tile<T, CH, kT>(slot(st, 1), p.mode_dt, dtg, p.sdt, b, d0, t0, tk, p.dim);
    if (zg) load_io_tile<T, CH, kT>(slot(st, 2), mode_z, zg, p.sz, b, d0, t0, tk, p.dim);
    cp_async_commit();
  };

  BCPrefetch<T, NS, CH, kT> pre;
  pre.load(p, b, 0, min(kT, p.seqlen));
  pre.store(bcs, p);
  issue(0);

  for (int k = 0; k < ntiles; ++k) {
    const int st = k & 1;
    const int t0 = k * kT, tk = min(kT, p.seqlen - t0);
    if (k + 1 < ntiles) {
      issue(k + 1);
      pre.load(p, b, t0 + kT, min(kT, p.seqlen - t0 - kT));
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    T* us = slot(st, 0);
    const T* ds = slot(st, 1);
    const T* zs = slot(st, 2);
    const float* bc = bcs + st * kT * 2 * NS;
    const bool has_z = zg != nullptr;
    const bool sp = p.softplus != 0;
    if constexpr (!ACC && !ZOH) {
      if (use_pow)
        compute_tile<T, NS, CH, kT, ACC, ZOH, true>(us, ds, zs, p.mode_u, p.mode_dt, mode_z, has_z, bc, tk, h, Al2, Aval,
                                                invA, bias, Dd, sp, p.z_mode, tid);
      else
        compute_tile<T, NS, CH, kT, ACC, ZOH, false>(us, ds, zs, p.mode_u, p.mode_dt, mode_z, has_z, bc, tk, h, Al2,
                                                 Aval, invA, bias, Dd, sp, p.z_mode, tid);
    } else {
      compute_tile<T, NS, CH, kT, ACC, ZOH, false>(us, ds, zs, p.mode_u, p.mode_dt, mode_z, has_z, bc, tk, h, Al2, Aval,
                                               invA, bias, Dd, sp, p.z_mode, tid);
    }
    if (k + 1 < ntiles) pre.store(bcs + (st ^ 1) * kT * 2 * NS, p);
    __syncthreads();
    store_y_tile<T, CH, kT>(us, p.mode_u, p.mode_y, yg, p.sy, b, d0, t0, tk, p.dim);
    __syncthreads();
  }

  if (p.hT && dvalid) {
#pragma unroll
    for (int n = 0; n < NS; ++n)
      if (n < p.dstate) p.hT[((int64_t)b * p.dim + d) * p.dstate + n] = h[n];
  }
}

template <typename T, int NS, int CH, int kT, bool ACC, bool ZOH>
hxm_status launch(const Params& p, cudaStream_t stream) {
  using S = Smem<T, CH, kT>;
  const size_t smem = sizeof(T) * 2 * 3 * S::kSlot + sizeof(float) * 2 * kT * 2 * NS;
  auto kern = scan_fwd_kernel<T, NS, CH, kT, ACC, ZOH>;
  if (smem > 48 * 1024) HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dim + CH - 1) / CH, p.batch);
  kern<<<grid, CH, smem, stream>>>(p);
  return check_launch("hxm_selective_scan_fwd");
}

// Launch-shape tuning knobs: HXM_SCAN_CH = 32|64 channels per CTA,
// HXM_SCAN_T = 32|64 timesteps per staged tile.  Unset = automatic choice.
int env_knob(const char* name);

template <typename T, int NS, bool ACC, bool ZOH>
hxm_status pick_ch(const Params& p, cudaStream_t stream, int num_sms) {
  // Choose the CTA width whose CTA count fills the SMs most evenly.
  auto eff = [&](int ch) {
    const double ctas = (double)((p.dim + ch - 1) / ch) * p.batch;
    const double per_sm = ctas / num_sms;
    return per_sm / std::ceil(per_sm) * ((double)p.dim / (((p.dim + ch - 1) / ch) * ch));
  };
  int ch = env_knob("HXM_SCAN_CH");
  if (ch != 32 && ch != 64) ch = (eff(64) >= eff(32) - 0.02) ? 64 : 32;
  int tt = env_knob("HXM_SCAN_T");
  if (tt != 32 && tt != 64) tt = 32;
  if constexpr (NS <= 16) {
    if (tt == 64)
      return ch == 64 ? launch<T, NS, 64, 64, ACC, ZOH>(p, stream) : launch<T, NS, 32, 64, ACC, ZOH>(p, stream);
  }
  return ch == 64 ? launch<T, NS, 64, 32, ACC, ZOH>(p, stream) : launch<T, NS, 32, 32, ACC, ZOH>(p, stream);
}

template <typename T, bool ACC, bool ZOH>
hxm_status pick_ns(const Params& p, cudaStream_t stream, int num_sms) {
  if (p.dstate <= 16) return pick_ch<T, 16, ACC, ZOH>(p, stream, num_sms);
  if (p.dstate <= 32) return pick_ch<T, 32, ACC, ZOH>(p, stream, num_sms);
  return pick_ch<T, 64, ACC, ZOH>(p, stream, num_sms);
}

// Explicitly instantiated in scan_inst_*.cu (one translation unit each).
hxm_status dispatch_f32_euler(const Params& p, cudaStream_t s, int num_sms);
hxm_status dispatch_f32_zoh(const Params& p, cudaStream_t s, int num_sms);
hxm_status dispatch_bf16_euler(const Params& p, cudaStream_t s, int num_sms);
hxm_status dispatch_bf16_zoh(const Params& p, cudaStream_t s, int num_sms);

}  // namespace scan
}  // namespace hxm
