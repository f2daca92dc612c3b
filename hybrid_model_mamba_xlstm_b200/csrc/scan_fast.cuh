// scan_fast.cuh — selective-scan kernel for the dominant layout (sm_100a).
//
// Covers dstate <= 16 in two layouts (16-byte aligned rows):
//   time-major:    u / delta / z / y unit time stride ((batch, dim, seqlen)
//                  memory), B, C unit time stride ((batch, dstate, seqlen));
//   channel-major: u / delta / z / y unit channel stride ((batch, seqlen, dim)
//                  memory, views with any row stride, e.g. the x / z halves of
//                  one in_proj output), B, C unit state stride ((batch, seqlen,
//                  dstate), e.g. column slices of the x_proj output).
// Every other layout runs the generic kernel of scan_kernel.cuh.
//
// Per CTA: CH channels of one batch row.  Per tile of kT steps, cp.async
// stages the u / delta / z rows and the raw bf16/fp32 B, C rows (double
// buffered); one cooperative pass converts B, C to an fp32 [t][B0..15 C0..15]
// table read with broadcast LDS.128.  Each thread runs one channel's 16
// states in 8 packed fp32x2 registers (FFMA2/FMUL2), the powers
// r^1..r^16 of r = exp(delta*A[0]) come from a depth-4 product tree when
// A[d, n] = (n+1)*A[d, 0] (checked per warp on the device), otherwise one
// exp per state.
#pragma once

#include "scan_kernel.cuh"

namespace hxm {
namespace scan {

template <typename T, int CH, int kT>
struct FastSmem {
  static constexpr int kPad = 16 / sizeof(T);
  static constexpr int kTP = kT + kPad;                        // io row pitch (elements)
  static constexpr int kIoSlot = CH * kTP;                     // one tensor tile
  static constexpr int kBcRaw = 32 * kTP;                      // raw B, C rows [32][kTP]
  static constexpr size_t kStageBytes = sizeof(T) * (3 * kIoSlot + kBcRaw);
  static constexpr size_t kBytes = 2 * kStageBytes + sizeof(float) * kT * 32;
};

HXM_DEV float2 f2(float a) { return make_float2(a, a); }

// State update of one step.  h[q] holds states (2q, 2q+1).  `r` = exp(delta*A[0])
// (POW) or delta (general path: exponents formed here).  Returns sum_n C_n h_n.
template <bool ZOH, bool POW>
HXM_DEV float fast_step(float r, float dl, float du, float u, const float* __restrict__ bc, float2 (&h)[8],
                        const float* __restrict__ Arow) {
  const float4* b4 = reinterpret_cast<const float4*>(bc);
  const float4* c4 = reinterpret_cast<const float4*>(bc + 16);
  float2 ya = make_float2(0.f, 0.f), yb = make_float2(0.f, 0.f);
  if (POW) {
    // r^1..r^16: one FMUL and seven FMUL2 (pairs (r^2k+1, r^2k+2) from the pairs before)
    const float r2 = r * r;
    float2 pw[8];
    pw[0] = make_float2(r, r2);
    pw[1] = __fmul2_rn(f2(r2), pw[0]);   // r^3, r^4
    pw[2] = __fmul2_rn(f2(pw[1].y), pw[0]);  // r^5, r^6
    pw[3] = __fmul2_rn(f2(pw[1].y), pw[1]);  // r^7, r^8
#pragma unroll
    for (int q = 0; q < 4; ++q) pw[4 + q] = __fmul2_rn(f2(pw[3].y), pw[q]);  // r^9 .. r^16
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 bb = b4[q], cc = c4[q];
      const float2 w0 = __fmul2_rn(f2(du), make_float2(bb.x, bb.y));
      const float2 w1 = __fmul2_rn(f2(du), make_float2(bb.z, bb.w));
      h[2 * q] = __ffma2_rn(pw[2 * q], h[2 * q], w0);
      h[2 * q + 1] = __ffma2_rn(pw[2 * q + 1], h[2 * q + 1], w1);
      ya = __ffma2_rn(make_float2(cc.x, cc.y), h[2 * q], ya);
      yb = __ffma2_rn(make_float2(cc.z, cc.w), h[2 * q + 1], yb);
    }
  } else {
    // general A: one exp per state; Arow = A[d, :] * log2(e) in shared memory
    const float4* a4 = reinterpret_cast<const float4*>(Arow);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 bb = b4[q], cc = c4[q], aa = a4[q];
      const float av[4] = {aa.x, aa.y, aa.z, aa.w};
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
      float dA[4], bbar[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x = dl * av[j];  // delta*A*log2(e)
        dA[j] = ex2_approx(x);
        if (ZOH) {
          // Bbar = (exp(dA)-1)/A * B, or delta*B when |delta*A| < 0.01
          const float xa = x * kLn2;
          bbar[j] = (fabsf(xa) < 0.01f) ? du * bv[j] : (dA[j] - 1.f) * (dl / xa) * bv[j] * u;
        } else {
          bbar[j] = du * bv[j];
        }
      }
      h[2 * q] = __ffma2_rn(make_float2(dA[0], dA[1]), h[2 * q], make_float2(bbar[0], bbar[1]));
      h[2 * q + 1] = __ffma2_rn(make_float2(dA[2], dA[3]), h[2 * q + 1], make_float2(bbar[2], bbar[3]));
      ya = __ffma2_rn(make_float2(cc.x, cc.y), h[2 * q], ya);
      yb = __ffma2_rn(make_float2(cc.z, cc.w), h[2 * q + 1], yb);
    }
  }
  const float2 ys = __fadd2_rn(ya, yb);
  return ys.x + ys.y;
}

// 8 steps of one channel from a staged tile: time-major rows [CH][kTP] (one
// 16-byte load) or channel-major rows [kT][CH] (8 conflict-free 2-byte loads).
template <typename T, int CH, int kT, bool CM>
HXM_DEV void tile_read8(const T* slot, int tid, int tt, float (&v)[8]) {
  if (CM) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32<T>(slot[(tt + j) * CH + tid]);
  } else {
    read8<T, CH, kT>(slot + tid * FastSmem<T, CH, kT>::kTP, kTimeMaj, 0, tt, v);
  }
}
template <typename T, int CH, int kT, bool CM>
HXM_DEV void tile_write8(T* slot, int tid, int tt, const float (&v)[8]) {
  if (CM) {
#pragma unroll
    for (int j = 0; j < 8; ++j) slot[(tt + j) * CH + tid] = from_f32<T>(v[j]);
  } else {
    write8<T, CH, kT>(slot + tid * FastSmem<T, CH, kT>::kTP, kTimeMaj, 0, tt, v);
  }
}

template <typename T, int CH, int kT, bool POW, int ZMODE, bool SP, bool MASK, bool CM>
HXM_DEV void fast_tile(T* us, const T* ds, const T* zs, const float* __restrict__ bc, int tk, float2 (&h)[8],
                       float a0l2, const float* Arow, float bias, float Dd, int tid) {
#pragma unroll 1
  for (int tt = 0; tt < kT; tt += 8) {
    float uv[8], dv[8], zv[8], yv[8];
    tile_read8<T, CH, kT, CM>(us, tid, tt, uv);
    tile_read8<T, CH, kT, CM>(ds, tid, tt, dv);
    if (ZMODE != 0) tile_read8<T, CH, kT, CM>(zs, tid, tt, zv);
    // phase A: the per-step scalar work of all 8 steps (independent, overlappable)
    float dl[8], du[8], rr[8], gz[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float x = dv[j] + bias;
      if (SP) x = softplus<false>(x);
      if (MASK) x = (tt + j < tk) ? x : 0.f;  // steps past the end leave h unchanged
      dl[j] = x;
      du[j] = x * uv[j];
      rr[j] = POW ? ex2_approx(x * a0l2) : x;
      gz[j] = ZMODE == 2 ? zv[j] * sigmoid<false>(zv[j]) : (ZMODE == 1 ? zv[j] : 1.f);
    }
    // phase B: the recurrence (short dependency chain through h)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float yy = fast_step<false, POW>(rr[j], dl[j], du[j], uv[j], bc + (tt + j) * 32, h, Arow);
      yv[j] = ZMODE == 0 ? fmaf(Dd, uv[j], yy) : fmaf(Dd, uv[j], yy) * gz[j];
    }
    tile_write8<T, CH, kT, CM>(us, tid, tt, yv);
  }
}

// Time segments: blockIdx.z = segment s of p.nseg (steps [tb, te)); a segment s > 0 starts
// from the carry h_s = exp(A * sum delta_{s-1}) . h_{s-1} + E_{s-1} of the earlier segments'
// zero-start end states E and delta sums, which scan_fast_state_kernel wrote to p.seg_ws.
template <typename T, int CH, int kT, int ZMODE, bool SP, bool CM>
__global__ void __launch_bounds__(CH) scan_fast_kernel(const Params p) {
  using S = FastSmem<T, CH, kT>;
  constexpr int kE = 16 / sizeof(T);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* bcf = reinterpret_cast<float*>(smem_raw + 2 * S::kStageBytes);  // [kT][32] fp32
  __shared__ __align__(16) float Ash[CH * 16];                             // A[d, :] * log2(e)

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * CH;
  const int d = d0 + tid;
  const bool dvalid = d < p.dim;
  const int dc = dvalid ? d : 0;
  const int seg = blockIdx.z;
  const int tb = p.nseg > 1 ? seg * p.seg_len : 0;
  const int te = p.nseg > 1 ? min(p.seqlen, tb + p.seg_len) : p.seqlen;

  bool pattern = true;
  const float a0 = p.A[(int64_t)dc * p.sA[0]];
  float2 h[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float hv[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = 2 * q + j;
      const float a = n < p.dstate ? p.A[(int64_t)dc * p.sA[0] + (int64_t)n * p.sA[1]] : 0.f;
      Ash[tid * 16 + n] = a * kLog2e;
      if (n < p.dstate && a != a0 * (float)(n + 1)) pattern = false;
      hv[j] = (p.h0 && dvalid && n < p.dstate) ? p.h0[((int64_t)b * p.dim + d) * p.dstate + n] : 0.f;
    }
    h[q] = make_float2(hv[0], hv[1]);
  }
  const bool use_pow = __all_sync(0xffffffffu, pattern);
  const float a0l2 = a0 * kLog2e;
  if (seg > 0) {
    // carry into this segment from the earlier segments' zero-start summaries
    const float* ws = p.seg_ws + ((int64_t)b * p.dim + dc) * (p.nseg - 1) * 17;
    for (int s2 = 0; s2 < seg; ++s2) {
      const float sdl = ws[s2 * 17 + 16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float2 P = make_float2(ex2_approx(Ash[tid * 16 + 2 * q] * sdl), ex2_approx(Ash[tid * 16 + 2 * q + 1] * sdl));
        h[q] = __ffma2_rn(P, h[q], make_float2(ws[s2 * 17 + 2 * q], ws[s2 * 17 + 2 * q + 1]));
      }
    }
  }
  const float Dd = (p.D && dvalid) ? p.D[d] : 0.f;
  const float bias = (p.bias && dvalid) ? p.bias[d] : 0.f;
  const bool has_z = ZMODE != 0;

  // per-thread global row pointers (time-major rows)
  const T* ug = static_cast<const T*>(p.u) + b * p.su[0];
  const T* dtg = static_cast<const T*>(p.dt) + b * p.sdt[0];
  const T* zg = has_z ? static_cast<const T*>(p.z) + b * p.sz[0] : nullptr;
  const T* Bg = static_cast<const T*>(p.B) + b * p.sB[0];
  const T* Cg = static_cast<const T*>(p.C) + b * p.sC[0];
  T* yg = static_cast<T*>(p.y) + b * p.sy[0];
  const int ntiles = (te - tb + kT - 1) / kT;

  auto stage_ptr = [&](int st) { return reinterpret_cast<T*>(smem_raw + st * S::kStageBytes); };
  // Whole tiles of a CTA whose channels and states all exist take a lean path: the thread's
  // copies sit at fixed row / step offsets from one base pointer per tensor, so a tile costs
  // one address add per 16-byte copy and no bounds arithmetic (measured at 8 x 32768 x 4096,
  // time-major: 5.45 -> 5.12 ms).
  const bool lean = d0 + CH <= p.dim && p.dstate == 16;
  auto issue = [&](int k) {
    T* base = stage_ptr(k & 1);
    const int t0 = tb + k * kT, tk = min(kT, te - t0);
    constexpr int kChunks = kT / kE;
    if (CM && lean && tk == kT) {
      // [kT][CH] step rows: thread = one 16-byte channel group of every (CH / kE)-th step row
      constexpr int kRowChunks = CH / kE, kStepStep = CH / kRowChunks;
      const int lt = tid / kRowChunks, lc = (tid % kRowChunks) * kE;
#pragma unroll
      for (int which = 0; which < 3; ++which) {
        if (which == 2 && !has_z) break;
        const T* g = which == 0 ? ug : (which == 1 ? dtg : zg);
        const int64_t st = which == 0 ? p.su[1] : (which == 1 ? p.sdt[1] : p.sz[1]);
        const T* src = g + (int64_t)(t0 + lt) * st + d0 + lc;
        T* dst = base + which * S::kIoSlot + lt * CH + lc;
#pragma unroll
        for (int i = 0; i < kT * kRowChunks / CH; ++i)
          cp_async16(dst + i * kStepStep * CH, src + (int64_t)i * kStepStep * st, 16);
      }
      // raw B, C step rows [kT][B0..15 C0..15]
      constexpr int kBcChunks = 32 / kE, kBcStep = CH / kBcChunks;
      const int bt = tid / kBcChunks, bn = (tid % kBcChunks) * kE;
      const T* bsrc = bn < 16 ? Bg + (int64_t)(t0 + bt) * p.sB[1] + bn : Cg + (int64_t)(t0 + bt) * p.sC[1] + (bn - 16);
      const int64_t bst = bn < 16 ? p.sB[1] : p.sC[1];
      T* raw = base + 3 * S::kIoSlot + bt * 32 + bn;
#pragma unroll
      for (int i = 0; i < kT * kBcChunks / CH; ++i) cp_async16(raw + i * kBcStep * 32, bsrc + (int64_t)i * kBcStep * bst, 16);
      cp_async_commit();
      return;
    }
    if (!CM && lean && tk == kT) {
      constexpr int kRowStep = CH / kChunks;  // rows between one thread's consecutive copies
      const int lr = tid / kChunks, lt = (tid % kChunks) * kE;
#pragma unroll
      for (int which = 0; which < 3; ++which) {
        if (which == 2 && !has_z) break;
        const T* g = which == 0 ? ug : (which == 1 ? dtg : zg);
        const int64_t sd = which == 0 ? p.su[2] : (which == 1 ? p.sdt[2] : p.sz[2]);
        const T* src = g + (int64_t)(d0 + lr) * sd + t0 + lt;
        T* dst = base + which * S::kIoSlot + lr * S::kTP + lt;
#pragma unroll
        for (int i = 0; i < kChunks; ++i) cp_async16(dst + i * kRowStep * S::kTP, src + (int64_t)i * kRowStep * sd, 16);
      }
      T* raw = base + 3 * S::kIoSlot;  // B rows 0..15, C rows 16..31
#pragma unroll
      for (int i = 0; i < 32 * kChunks / CH; ++i) {
        const int row = lr + i * kRowStep, n = row % 16;
        const T* g = row >= 16 ? Cg + (int64_t)n * p.sC[2] : Bg + (int64_t)n * p.sB[2];
        cp_async16(raw + row * S::kTP + lt, g + t0 + lt, 16);
      }
      cp_async_commit();
      return;
    }
    // u, delta, z rows
#pragma unroll 1
    for (int which = 0; which < 3; ++which) {
      if (which == 2 && !has_z) break;
      const T* g = which == 0 ? ug : (which == 1 ? dtg : zg);
      const int64_t sd = which == 0 ? p.su[2] : (which == 1 ? p.sdt[2] : p.sz[2]);
      T* slot = base + which * S::kIoSlot;
      if (CM) {
        // [kT][CH]: step rows of CH channels (sd = time stride)
        const int64_t st = which == 0 ? p.su[1] : (which == 1 ? p.sdt[1] : p.sz[1]);
        constexpr int kRowChunks = CH / kE;
        for (int c = tid; c < kT * kRowChunks; c += CH) {
          const int t = c / kRowChunks, ch = (c % kRowChunks) * kE;
          const int valid = (t < tk) ? max(0, min(kE, p.dim - (d0 + ch))) : 0;
          const T* src = valid > 0 ? g + (int64_t)(t0 + t) * st + d0 + ch : g;
          cp_async16(slot + t * CH + ch, src, valid * (int)sizeof(T));
        }
      } else {
        for (int c = tid; c < CH * kChunks; c += CH) {
          const int ch = c / kChunks, t = (c % kChunks) * kE;
          const int dd = d0 + ch;
          const int valid = (dd < p.dim) ? max(0, min(kE, tk - t)) : 0;
          const T* src = valid > 0 ? g + (int64_t)dd * sd + t0 + t : g;
          cp_async16(slot + ch * S::kTP + t, src, valid * (int)sizeof(T));
        }
      }
    }
    T* raw = base + 3 * S::kIoSlot;
    if (CM) {
      // raw B, C step rows [kT][B0..15 C0..15]
      constexpr int kRowChunks = 32 / kE;
      for (int c = tid; c < kT * kRowChunks; c += CH) {
        const int t = c / kRowChunks, n = (c % kRowChunks) * kE;
        const int which = n / 16, n0 = n % 16;
        const int valid = (t < tk) ? max(0, min(kE, p.dstate - n0)) : 0;
        const T* g = which ? Cg + (int64_t)(t0 + t) * p.sC[1] + n0 : Bg + (int64_t)(t0 + t) * p.sB[1] + n0;
        cp_async16(raw + t * 32 + n, valid > 0 ? g : Bg, valid * (int)sizeof(T));
      }
    } else {
      // raw B, C rows [2][16][kT]
      for (int c = tid; c < 2 * 16 * kChunks; c += CH) {
        const int row = c / kChunks, t = (c % kChunks) * kE;
        const int which = row / 16, n = row % 16;
        const int valid = (n < p.dstate) ? max(0, min(kE, tk - t)) : 0;
        const T* g = which ? Cg + (int64_t)n * p.sC[2] : Bg + (int64_t)n * p.sB[2];
        cp_async16(raw + row * S::kTP + t, valid > 0 ? g + t0 + t : Bg, valid * (int)sizeof(T));
      }
    }
    cp_async_commit();
  };

  issue(0);
  for (int k = 0; k < ntiles; ++k) {
    const int st = k & 1;
    const int t0 = tb + k * kT, tk = min(kT, te - t0);
    cp_async_wait<0>();
    __syncthreads();  // tile k staged; previous tile's y stored and bc table consumed
    if (k + 1 < ntiles) issue(k + 1);
    // B, C rows -> fp32 [t][32] table: a thread reads 8 steps of one row with
    // one 16-byte load (padded rows: conflict-free) and writes them down the
    // column (lanes = 32 distinct columns: conflict-free).
    {
      const T* raw = stage_ptr(st) + 3 * S::kIoSlot;
      for (int c = tid; c < 32 * (kT / 8); c += CH) {
        float v[8];
        if (CM) {
          // step rows are already [t][32]: convert 8 consecutive values in place
          read8<T, CH, kT>(raw + c * 8, kTimeMaj, 0, 0, v);
          float4* dst = reinterpret_cast<float4*>(bcf + c * 8);
          dst[0] = make_float4(v[0], v[1], v[2], v[3]);
          dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
          const int col = c % 32, t8 = (c / 32) * 8;
          read8<T, CH, kT>(raw + col * S::kTP, kTimeMaj, 0, t8, v);
#pragma unroll
          for (int j = 0; j < 8; ++j) bcf[(t8 + j) * 32 + col] = v[j];
        }
      }
    }
    __syncthreads();
    T* us = stage_ptr(st);
    const T* ds = us + S::kIoSlot;
    const T* zs = us + 2 * S::kIoSlot;
    const float* Arow = Ash + tid * 16;
    if (tk == kT) {
      if (use_pow) fast_tile<T, CH, kT, true, ZMODE, SP, false, CM>(us, ds, zs, bcf, tk, h, a0l2, Arow, bias, Dd, tid);
      else fast_tile<T, CH, kT, false, ZMODE, SP, false, CM>(us, ds, zs, bcf, tk, h, a0l2, Arow, bias, Dd, tid);
    } else {
      if (use_pow) fast_tile<T, CH, kT, true, ZMODE, SP, true, CM>(us, ds, zs, bcf, tk, h, a0l2, Arow, bias, Dd, tid);
      else fast_tile<T, CH, kT, false, ZMODE, SP, true, CM>(us, ds, zs, bcf, tk, h, a0l2, Arow, bias, Dd, tid);
    }
    __syncthreads();
    // y tile (in u's slot) -> global, 16-byte stores along each channel row
    if (CM) {
      constexpr int kRowChunks = CH / kE;
      for (int c = tid; c < kT * kRowChunks; c += CH) {
        const int t = c / kRowChunks, ch = (c % kRowChunks) * kE;
        const int nv = min(kE, p.dim - (d0 + ch));
        if (t >= tk || nv <= 0) continue;
        const T* src = us + t * CH + ch;
        T* dst = yg + (int64_t)(t0 + t) * p.sy[1] + d0 + ch;
        if (nv == kE) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        else
          for (int j = 0; j < nv; ++j) dst[j] = src[j];
      }
    } else {
      constexpr int kChunks = kT / kE;
      for (int c = tid; c < CH * kChunks; c += CH) {
        const int ch = c / kChunks, t = (c % kChunks) * kE;
        const int dd = d0 + ch;
        if (dd >= p.dim || t >= tk) continue;
        const T* src = us + ch * S::kTP + t;
        T* dst = yg + (int64_t)dd * p.sy[2] + t0 + t;
        if (t + kE <= tk) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        else
          for (int j = 0; j < tk - t; ++j) dst[j] = src[j];
      }
    }
  }

  if (p.hT && dvalid && te == p.seqlen) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (2 * q < p.dstate) p.hT[((int64_t)b * p.dim + d) * p.dstate + 2 * q] = h[q].x;
      if (2 * q + 1 < p.dstate) p.hT[((int64_t)b * p.dim + d) * p.dstate + 2 * q + 1] = h[q].y;
    }
  }
}

// State-only pass over the first nseg - 1 segments (whole tiles): each (channel, segment) runs
// the recurrence from a zero state over its steps — no readout, no z, no y — and records the
// state it reaches and its sum of delta (after softplus) in p.seg_ws.  Same staging as the
// main kernel minus z and C.
template <typename T, int CH, int kT, bool SP, bool CM>
__global__ void __launch_bounds__(CH) scan_fast_state_kernel(const Params p) {
  using S = FastSmem<T, CH, kT>;
  constexpr int kE = 16 / sizeof(T);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* bcf = reinterpret_cast<float*>(smem_raw + 2 * S::kStageBytes);  // [kT][32] fp32 (B half used)
  __shared__ __align__(16) float Ash[CH * 16];

  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int d0 = blockIdx.x * CH;
  const int d = d0 + tid;
  const bool dvalid = d < p.dim;
  const int dc = dvalid ? d : 0;
  const int seg = blockIdx.z;  // < nseg - 1: full tiles only
  const int tb = seg * p.seg_len;
  const int ntiles = p.seg_len / kT;

  bool pattern = true;
  const float a0 = p.A[(int64_t)dc * p.sA[0]];
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const float a = n < p.dstate ? p.A[(int64_t)dc * p.sA[0] + (int64_t)n * p.sA[1]] : 0.f;
    Ash[tid * 16 + n] = a * kLog2e;
    if (n < p.dstate && a != a0 * (float)(n + 1)) pattern = false;
  }
  const bool use_pow = __all_sync(0xffffffffu, pattern);
  const float a0l2 = a0 * kLog2e;
  const float bias = (p.bias && dvalid) ? p.bias[d] : 0.f;
  float2 h[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) h[q] = make_float2(0.f, 0.f);
  float sdl = 0.f;

  const T* ug = static_cast<const T*>(p.u) + b * p.su[0];
  const T* dtg = static_cast<const T*>(p.dt) + b * p.sdt[0];
  const T* Bg = static_cast<const T*>(p.B) + b * p.sB[0];
  auto stage_ptr = [&](int st) { return reinterpret_cast<T*>(smem_raw + st * S::kStageBytes); };
  const bool lean = d0 + CH <= p.dim && p.dstate == 16;  // whole tiles only here
  auto issue = [&](int k) {
    T* base = stage_ptr(k & 1);
    const int t0 = tb + k * kT;
    constexpr int kChunks = kT / kE;
    if (lean) {  // fixed per-thread offsets, one address add per 16-byte copy (see scan_fast_kernel)
      if (CM) {
        constexpr int kRowChunks = CH / kE, kStepStep = CH / kRowChunks;
        const int lt = tid / kRowChunks, lc = (tid % kRowChunks) * kE;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const T* g = which == 0 ? ug : dtg;
          const int64_t st = which == 0 ? p.su[1] : p.sdt[1];
          const T* src = g + (int64_t)(t0 + lt) * st + d0 + lc;
          T* dst = base + which * S::kIoSlot + lt * CH + lc;
#pragma unroll
          for (int i = 0; i < kT * kRowChunks / CH; ++i)
            cp_async16(dst + i * kStepStep * CH, src + (int64_t)i * kStepStep * st, 16);
        }
        constexpr int kBChunks = 16 / kE, kBStep = CH / kBChunks;  // B step rows [kT][B0..15]
        const int bt = tid / kBChunks, bn = (tid % kBChunks) * kE;
        if (kT * kBChunks >= CH || tid < kT * kBChunks) {
          T* raw = base + 3 * S::kIoSlot + bt * 32 + bn;
          const T* bsrc = Bg + (int64_t)(t0 + bt) * p.sB[1] + bn;
#pragma unroll
          for (int i = 0; i < (kT * kBChunks + CH - 1) / CH; ++i)
            cp_async16(raw + i * kBStep * 32, bsrc + (int64_t)i * kBStep * p.sB[1], 16);
        }
      } else {
        constexpr int kRowStep = CH / kChunks;
        const int lr = tid / kChunks, lt = (tid % kChunks) * kE;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const T* g = which == 0 ? ug : dtg;
          const int64_t sd = which == 0 ? p.su[2] : p.sdt[2];
          const T* src = g + (int64_t)(d0 + lr) * sd + t0 + lt;
          T* dst = base + which * S::kIoSlot + lr * S::kTP + lt;
#pragma unroll
          for (int i = 0; i < kChunks; ++i) cp_async16(dst + i * kRowStep * S::kTP, src + (int64_t)i * kRowStep * sd, 16);
        }
        if (16 * kChunks >= CH || tid < 16 * kChunks) {  // B rows [16][kT]
          T* raw = base + 3 * S::kIoSlot;
#pragma unroll
          for (int i = 0; i < (16 * kChunks + CH - 1) / CH; ++i) {
            const int n = lr + i * kRowStep;
            cp_async16(raw + n * S::kTP + lt, Bg + (int64_t)n * p.sB[2] + t0 + lt, 16);
          }
        }
      }
      cp_async_commit();
      return;
    }
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const T* g = which == 0 ? ug : dtg;
      T* slot = base + which * S::kIoSlot;
      if (CM) {
        const int64_t st = which == 0 ? p.su[1] : p.sdt[1];
        constexpr int kRowChunks = CH / kE;
        for (int c = tid; c < kT * kRowChunks; c += CH) {
          const int t = c / kRowChunks, ch = (c % kRowChunks) * kE;
          const int valid = max(0, min(kE, p.dim - (d0 + ch)));
          const T* src = valid > 0 ? g + (int64_t)(t0 + t) * st + d0 + ch : g;
          cp_async16(slot + t * CH + ch, src, valid * (int)sizeof(T));
        }
      } else {
        const int64_t sd = which == 0 ? p.su[2] : p.sdt[2];
        for (int c = tid; c < CH * kChunks; c += CH) {
          const int ch = c / kChunks, t = (c % kChunks) * kE;
          const int dd = d0 + ch;
          const int valid = dd < p.dim ? kE : 0;
          const T* src = valid > 0 ? g + (int64_t)dd * sd + t0 + t : g;
          cp_async16(slot + ch * S::kTP + t, src, valid * (int)sizeof(T));
        }
      }
    }
    T* raw = base + 3 * S::kIoSlot;
    if (CM) {  // B step rows [kT][B0..15]
      constexpr int kRowChunks = 16 / kE;
      for (int c = tid; c < kT * kRowChunks; c += CH) {
        const int t = c / kRowChunks, n0 = (c % kRowChunks) * kE;
        const int valid = max(0, min(kE, p.dstate - n0));
        cp_async16(raw + t * 32 + n0, valid > 0 ? Bg + (int64_t)(t0 + t) * p.sB[1] + n0 : Bg, valid * (int)sizeof(T));
      }
    } else {  // B rows [16][kT]
      for (int c = tid; c < 16 * kChunks; c += CH) {
        const int n = c / kChunks, t = (c % kChunks) * kE;
        const int valid = n < p.dstate ? kE : 0;
        cp_async16(raw + n * S::kTP + t, valid > 0 ? Bg + (int64_t)n * p.sB[2] + t0 + t : Bg,
                   valid * (int)sizeof(T));
      }
    }
    cp_async_commit();
  };

  issue(0);
  for (int k = 0; k < ntiles; ++k) {
    const int st = k & 1;
    cp_async_wait<0>();
    __syncthreads();
    if (k + 1 < ntiles) issue(k + 1);
    {  // B rows -> fp32 [t][32] table (columns 0..15)
      const T* raw = stage_ptr(st) + 3 * S::kIoSlot;
      for (int c = tid; c < 16 * (kT / 8); c += CH) {
        float v[8];
        if (CM) {
          const int t = c / 2, n8 = (c % 2) * 8;
          read8<T, CH, kT>(raw + t * 32 + n8, kTimeMaj, 0, 0, v);
          float4* dst = reinterpret_cast<float4*>(bcf + t * 32 + n8);
          dst[0] = make_float4(v[0], v[1], v[2], v[3]);
          dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
          const int col = c % 16, t8 = (c / 16) * 8;
          read8<T, CH, kT>(raw + col * S::kTP, kTimeMaj, 0, t8, v);
#pragma unroll
          for (int j = 0; j < 8; ++j) bcf[(t8 + j) * 32 + col] = v[j];
        }
      }
    }
    __syncthreads();
    const T* us = stage_ptr(st);
    const T* ds = us + S::kIoSlot;
#pragma unroll 1
    for (int tt = 0; tt < kT; tt += 8) {
      float uv[8], dv[8];
      tile_read8<T, CH, kT, CM>(us, tid, tt, uv);
      tile_read8<T, CH, kT, CM>(ds, tid, tt, dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float x = dv[j] + bias;
        if (SP) x = softplus<false>(x);
        sdl += x;
        const float du = x * uv[j];
        const float4* b4 = reinterpret_cast<const float4*>(bcf + (tt + j) * 32);
        if (use_pow) {
          const float r = ex2_approx(x * a0l2);
          const float r2 = r * r, r4 = r2 * r2, r8 = r4 * r4;
          float2 pw[8];
          pw[0] = make_float2(r, r2);
          pw[1] = make_float2(r2 * r, r4);
          pw[2] = __fmul2_rn(f2(r4), pw[0]);
          pw[3] = __fmul2_rn(f2(r4), pw[1]);
#pragma unroll
          for (int q = 0; q < 4; ++q) pw[4 + q] = __fmul2_rn(f2(r8), pw[q]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 bb = b4[q];
            h[2 * q] = __ffma2_rn(pw[2 * q], h[2 * q], __fmul2_rn(f2(du), make_float2(bb.x, bb.y)));
            h[2 * q + 1] = __ffma2_rn(pw[2 * q + 1], h[2 * q + 1], __fmul2_rn(f2(du), make_float2(bb.z, bb.w)));
          }
        } else {
          const float4* a4 = reinterpret_cast<const float4*>(Ash + tid * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 bb = b4[q], aa = a4[q];
            h[2 * q] = __ffma2_rn(make_float2(ex2_approx(x * aa.x), ex2_approx(x * aa.y)), h[2 * q],
                                  __fmul2_rn(f2(du), make_float2(bb.x, bb.y)));
            h[2 * q + 1] = __ffma2_rn(make_float2(ex2_approx(x * aa.z), ex2_approx(x * aa.w)), h[2 * q + 1],
                                      __fmul2_rn(f2(du), make_float2(bb.z, bb.w)));
          }
        }
      }
    }
  }
  if (dvalid) {
    float* ws = p.seg_ws + (((int64_t)b * p.dim + d) * (p.nseg - 1) + seg) * 17;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      ws[2 * q] = h[q].x;
      ws[2 * q + 1] = h[q].y;
    }
    ws[16] = sdl;
  }
}

template <typename T, int CH, int kT, int ZMODE, bool SP, bool CM>
hxm_status launch_fast(const Params& p, cudaStream_t stream) {
  using S = FastSmem<T, CH, kT>;
  const size_t smem = S::kBytes;
  if (p.nseg > 1) {
    auto skern = scan_fast_state_kernel<T, CH, kT, SP, CM>;
    if (smem > 48 * 1024 - sizeof(float) * CH * 16)
      HXM_CUDA_TRY(cudaFuncSetAttribute(skern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 sgrid((p.dim + CH - 1) / CH, p.batch, p.nseg - 1);
    skern<<<sgrid, CH, smem, stream>>>(p);
    hxm_status s = check_launch("hxm_selective_scan_fwd (segment states)");
    if (s != HXM_OK) return s;
  }
  auto kern = scan_fast_kernel<T, CH, kT, ZMODE, SP, CM>;
  if (smem > 48 * 1024 - sizeof(float) * CH * 16)
    HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dim + CH - 1) / CH, p.batch, p.nseg > 1 ? p.nseg : 1);
  kern<<<grid, CH, smem, stream>>>(p);
  return check_launch("hxm_selective_scan_fwd (fast)");
}

// Which layout the fast kernel can run this request in: 1 time-major,
// 2 channel-major, 0 neither (generic kernel).
inline int fast_layout(const Params& p, size_t esize) {
  if (p.dstate > 16) return 0;
  const int64_t e16 = 16 / (int64_t)esize;
  auto bc_ok = [&](const void* ptr, const int64_t* s, int unit) {
    const int o1 = unit == 1 ? 2 : 1;
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && s[unit] == 1 && s[0] % e16 == 0 && s[o1] % e16 == 0;
  };
  for (int mode : {(int)kTimeMaj, (int)kChanMaj}) {
    if (p.mode_u != mode || p.mode_dt != mode || p.mode_y != mode) continue;
    if (p.z && p.mode_z != mode) continue;
    const int unit = mode == kTimeMaj ? 1 : 2;  // B, C: unit time stride / unit state stride
    if (bc_ok(p.B, p.sB, unit) && bc_ok(p.C, p.sC, unit)) return mode == kTimeMaj ? 1 : 2;
  }
  return 0;
}
inline bool fast_ok(const Params& p, size_t esize) { return fast_layout(p, esize) != 0; }

template <typename T, int CH, int kT, bool CM>
hxm_status pick_fast_modes_t(const Params& p, cudaStream_t stream) {
  const int zm = p.z ? p.z_mode : 0;
  if (p.softplus) {
    if (zm == 2) return launch_fast<T, CH, kT, 2, true, CM>(p, stream);
    if (zm == 1) return launch_fast<T, CH, kT, 1, true, CM>(p, stream);
    return launch_fast<T, CH, kT, 0, true, CM>(p, stream);
  }
  if (zm == 2) return launch_fast<T, CH, kT, 2, false, CM>(p, stream);
  if (zm == 1) return launch_fast<T, CH, kT, 1, false, CM>(p, stream);
  return launch_fast<T, CH, kT, 0, false, CM>(p, stream);
}
// Tile length: 32 steps in one pass; 16 with time segments (half the shared memory per CTA, so
// more of the segments' CTAs are resident: one row x 32768 x 4096 in 16 segments 1.08 ms vs
// 1.22 with 32-step tiles, four rows 3.47 vs 3.96; in one pass 32-step tiles are faster, 5.44
// vs 5.60 ms for eight rows).  HXM_SCAN_FAST_T = 16 | 32 overrides.
template <typename T, int CH, bool CM>
hxm_status pick_fast_modes(const Params& p, cudaStream_t stream) {
  int t = env_knob("HXM_SCAN_FAST_T");
  if (t != 16 && t != 32) t = p.nseg > 1 ? 16 : 32;
  if (t == 16) return pick_fast_modes_t<T, CH, 16, CM>(p, stream);  // segment lengths are multiples of 32
  return pick_fast_modes_t<T, CH, 32, CM>(p, stream);
}

// Time segments for the fast kernel: a small grid leaves most of the GPU idle (one thread per
// channel; e.g. one batch row of 4096 channels = 64 CTAs on 148 SMs), so the sequence is cut
// into 16 segments of >= 128 steps (a multiple of 32) that run in parallel after a state-only
// pass over the first 15 (about 40 % more work in all).  Measured on B200, x 32768 x 4096,
// 16-step tiles: one row 4.09 ms in one pass -> 1.08 ms in 16 segments; four rows 4.13 -> 3.47;
// eight rows (3.5 CTAs per SM) 5.44 in one pass against 6.74, so segments stop at 2.5 CTAs per
// SM.  With fewer segments the state pass itself stays occupancy-bound (one row: 1.99 ms with 4).
// Short sequences (the prefill's 256-2048-step pieces) run one pass: there the second launch and
// the pipeline fill of short segments cost more than the idle SMs, which the other layers'
// kernels of the wavefront occupy anyway (hybrid-350M prefill 31.1 ms one pass, 33.0 segmented).
// HXM_SCAN_NSEG forces a count (1 = one pass).
inline int fast_segments(const Params& p, int num_sms, int* seg_len) {
  const int ch = p.dim >= 64 ? 64 : 32;
  const int64_t ctas = (int64_t)((p.dim + ch - 1) / ch) * p.batch;
  int nseg = env_knob("HXM_SCAN_NSEG");
  if (nseg <= 0) nseg = (ctas * 2 < (int64_t)num_sms * 5 && p.seqlen >= 8192) ? 16 : 1;
  nseg = max(1, min(nseg, 16));
  int len = 0;
  while (nseg > 1) {
    len = ((p.seqlen + nseg - 1) / nseg + 31) / 32 * 32;
    if (len >= 128 || env_knob("HXM_SCAN_NSEG") > 0) break;
    nseg /= 2;
  }
  if (nseg > 1) nseg = (p.seqlen + len - 1) / len;  // segments actually covered
  *seg_len = nseg > 1 ? len : p.seqlen;
  return nseg > 1 ? nseg : 1;
}

// CTA width: 64 channels (two warps sharing one B, C table) unless the
// channel count is small; measured faster than 32 on B200 at every batch size
// of the 4096-channel workload (1..16 batch rows), despite the coarser
// CTA-per-SM balance.
template <typename T>
hxm_status pick_fast(const Params& p, cudaStream_t stream, int /*num_sms*/) {
  int ch = env_knob("HXM_SCAN_CH");
  if (ch != 32 && ch != 64) ch = p.dim >= 64 ? 64 : 32;
  if (fast_layout(p, sizeof(T)) == 2)
    return ch == 64 ? pick_fast_modes<T, 64, true>(p, stream) : pick_fast_modes<T, 32, true>(p, stream);
  return ch == 64 ? pick_fast_modes<T, 64, false>(p, stream) : pick_fast_modes<T, 32, false>(p, stream);
}

}  // namespace scan
}  // namespace hxm
