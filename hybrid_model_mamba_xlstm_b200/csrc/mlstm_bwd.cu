// mlstm_bwd.cu — element-wise and scan kernels of the chunkwise mLSTM
// backward (sm_100a).
//
// The reference's backward (TFLAFunction.backward,
// hybrid_xmamba/kernels/tfla/tfla_interface.py:52-81) re-runs the step loop
// tfla_forward_pytorch (:84-139) under autograd.  The chunkwise form used
// here: for a chunk of c steps and key channel j, b_t = sum_{s<=t} log f_s
// (inside the chunk), g = b_{c-1}, rho = g/2 and
//     Qs_t = q_t e^(b_t - rho),   Ks_s = k_s e^(log i_s + rho - b_s)
// so that q_t . (e^(b_t - b_s) i_s k_s) = Qs_t . Ks_s (intra-chunk) and the
// state entering the next chunk is  e^g C + e^rho Ks^T [v | 1]  (the
// normalizer n rides along as an extra column of ones).  The batched chunk
// GEMMs (S = Qs Ks^T, its gradients, the chunk-state increments) run as
// library GEMMs between these kernels:
//   prepare   q, k, log gates -> Qs, Ks, rho, e^rho, e^g per chunk
//   scan      exclusive chunk-level recurrences s' = diag(decay) s + x, run
//             forward for the states entering each chunk and in reverse for
//             the state adjoints leaving each chunk
//   finalize  dL/dQs, dL/dKs -> dq = e^(b - rho) dL/dQs,
//             dk = i e^(rho - b) dL/dKs, dlog_i = Ks . dL/dKs and
//             dlog_f_t = dg + sum_{s >= t in the chunk} (Qs . dL/dQs - Ks . dL/dKs)_s
// The loss sees the chunk's log f only through the in-chunk prefix sums b
// (gradient q_t dq_t - (i k)_t d(i k)_t at step t, the gate identity of decayed
// linear recurrences) and through the chunk total g, whose gradient dg is the
// inner product of the state leaving the chunk with its adjoint (an input).
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace mlstm_bwd {

struct Params {
  int batch, heads, seqlen, dqk, chunk, nch, gate_mode;
  const void* q;
  int64_t sq[3];
  const void* k;
  int64_t sk[3];
  const float* log_i;
  int64_t si[3];
  const float* log_f;
  int64_t sf[3];
  float *qs, *ks, *rho, *erho, *eg, *qd, *kd;
  __nv_bfloat16* planes;  // optional: hi / lo planes of qs, ks, qd, kd (8 planes of `plane` elements)
  int64_t plane;
  const float *dqs, *dks;
  const float* dg;
  float *dq, *dk, *dli, *dlf, *di;
};

// grid (batch*heads*nch, ceil(dqk/128)), block 128: thread = key channel j of one chunk
template <typename T>
__global__ void __launch_bounds__(128) prepare_kernel(const Params p) {
  const int j = blockIdx.y * 128 + threadIdx.x;
  if (j >= p.dqk) return;
  const int kc = blockIdx.x % p.nch, bh = blockIdx.x / p.nch;
  const int b = bh / p.heads, h = bh % p.heads;
  const int t0 = kc * p.chunk, tn = min(p.chunk, p.seqlen - t0);
  const int64_t jg = p.gate_mode ? j : 0;
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1] + jg;
  const float* li = p.log_i + b * p.si[0] + h * p.si[1] + jg;
  const T* q = static_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1] + j;
  const T* k = static_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1] + j;
  float g = 0.f;
  for (int s = 0; s < tn; ++s) g += lf[(int64_t)(t0 + s) * p.sf[2]];
  const float rho = 0.5f * g;
  const int64_t vo = ((int64_t)bh * p.nch + kc) * p.dqk + j;
  const float erho = expf(rho);
  p.rho[vo] = rho;
  p.erho[vo] = erho;
  p.eg[vo] = expf(g);
  const int64_t ro = ((int64_t)bh * p.nch + kc) * p.chunk * p.dqk + j;
  float bt = 0.f;
  for (int s = 0; s < p.chunk; ++s) {
    float qv = 0.f, kv = 0.f;
    if (s < tn) {
      const int64_t t = t0 + s;
      bt += lf[t * p.sf[2]];
      qv = to_f32<T>(q[t * p.sq[2]]) * expf(bt - rho);
      kv = to_f32<T>(k[t * p.sk[2]]) * expf(li[t * p.si[2]] + rho - bt);
    }
    const int64_t o = ro + (int64_t)s * p.dqk;
    if (p.qs) p.qs[o] = qv;
    if (p.ks) p.ks[o] = kv;
    if (p.qd) p.qd[o] = qv * erho;  // q e^b
    if (p.kd) p.kd[o] = kv * erho;  // i k e^(g - b)
    if (p.planes) {
      const float vals[4] = {qv, kv, qv * erho, kv * erho};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(vals[u]);
        p.planes[(2 * u) * p.plane + o] = hi;
        p.planes[(2 * u + 1) * p.plane + o] = __float2bfloat16_rn(vals[u] - __bfloat162float(hi));
      }
    }
  }
}

// q_scaled / k_scaled at element o: the fp32 arrays, or high + low from the split planes.
HXM_DEV float scaled_at(const Params& p, const float* arr, int which, int64_t o) {
  if (arr) return arr[o];
  return __bfloat162float(p.planes[(2 * which) * p.plane + o]) + __bfloat162float(p.planes[(2 * which + 1) * p.plane + o]);
}

// grid (batch*heads*nch, ceil(dqk/128)), block 128: the chunk's steps in reverse,
// b_t rebuilt from g = 2 rho; dlog_f = the chunk's dg plus the within-chunk
// suffix sum of the gate identity.  di (optional): the gradient
// with respect to the gate value i = e^(log_i), k . dL/d(i k), formed without
// dividing by i.
template <typename T>
__global__ void __launch_bounds__(128) finalize_kernel(const Params p) {
  const int j = blockIdx.y * 128 + threadIdx.x;
  if (j >= p.dqk) return;
  const int kc = blockIdx.x % p.nch, bh = blockIdx.x / p.nch;
  const int b = bh / p.heads, h = bh % p.heads;
  const int t0 = kc * p.chunk, tn = min(p.chunk, p.seqlen - t0);
  const int64_t jg = p.gate_mode ? j : 0;
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1] + jg;
  const float* li = p.log_i + b * p.si[0] + h * p.si[1] + jg;
  const T* k = static_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1] + j;
  const int64_t vo = ((int64_t)bh * p.nch + kc) * p.dqk + j;
  const float rho = p.rho[vo];
  float bt = 2.f * rho;  // b at the chunk's last real step
  const int64_t ro = ((int64_t)bh * p.nch + kc) * p.chunk * p.dqk + j;
  const int64_t oo = ((int64_t)bh * p.seqlen + t0) * p.dqk + j;
  float acc = p.dg[vo];
  for (int s = tn - 1; s >= 0; --s) {
    const int64_t t = t0 + s;
    const int64_t r = ro + (int64_t)s * p.dqk, o = oo + (int64_t)s * p.dqk;
    const float P = p.dqs[r], R = p.dks[r], Qv = scaled_at(p, p.qs, 0, r), Kv = scaled_at(p, p.ks, 1, r);
    p.dq[o] = expf(bt - rho) * P;
    const float ek = expf(rho - bt) * R;  // dL/d(i k)
    const float iv = expf(li[t * p.si[2]]);
    p.dk[o] = iv * ek;
    if (p.di) p.di[o] = to_f32<T>(k[t * p.sk[2]]) * ek;
    p.dli[o] = Kv * R;
    acc += Qv * P - Kv * R;
    // f at the sequence's first step multiplies the zero initial state: its
    // gradient is exactly zero (the identity's sum cancels to rounding there)
    p.dlf[o] = t == 0 ? 0.f : acc;
    bt -= lf[t * p.sf[2]];
  }
}

// one thread per (group, row, col) element, chunks in order (or reversed); the
// loads of 8 chunks are issued before their dependent updates, so a thread
// keeps 8 reads in flight instead of one load-store round trip per chunk
__global__ void __launch_bounds__(256) chunk_scan_kernel(float* __restrict__ x, const float* __restrict__ decay,
                                                         const float* __restrict__ scale, float* __restrict__ scaled,
                                                         __nv_bfloat16* __restrict__ shi, __nv_bfloat16* __restrict__ slo,
                                                         int64_t groups, int nch, int rows, int cols, int reverse) {
  constexpr int kB = 8;
  const int64_t rc = (int64_t)rows * cols;
  const int64_t e = blockIdx.x * 256ll + threadIdx.x;
  if (e >= groups * rc) return;
  const int64_t grp = e / rc, w = e % rc;
  const int r = (int)(w / cols);
  float* xp = x + grp * nch * rc + w;
  float* op = scaled ? scaled + grp * nch * rc + w : nullptr;
  const float* dp = decay ? decay + grp * nch * rows + r : nullptr;
  const float* sp = scale ? scale + grp * nch * rows + r : nullptr;
  float s = 0.f;
  for (int it0 = 0; it0 < nch; it0 += kB) {
    float y[kB], dc[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int it = it0 + u;
      const int kc = reverse ? nch - 1 - it : it;
      y[u] = it < nch ? xp[kc * rc] : 0.f;
      dc[u] = (it < nch && dp) ? dp[(int64_t)kc * rows] : 1.f;
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int it = it0 + u;
      if (it < nch) {
        const int kc = reverse ? nch - 1 - it : it;
        xp[kc * rc] = s;
        const float f = sp ? sp[(int64_t)kc * rows] : 1.f;
        if (op) op[kc * rc] = f * s;
        if (shi) {
          const int64_t o = grp * nch * rc + w + kc * rc;
          const __nv_bfloat16 hi = __float2bfloat16_rn(f * s);
          shi[o] = hi;
          if (slo) slo[o] = __float2bfloat16_rn(f * s - __bfloat162float(hi));
        }
        s = dc[u] * s + y[u];
      }
    }
  }
}

// The same with 4 adjacent columns of one row per thread (cols % 4 == 0, x
// 16-byte aligned): 16-byte loads and stores, one decay load per 4 columns.
__global__ void __launch_bounds__(256) chunk_scan4_kernel(float4* __restrict__ x, const float* __restrict__ decay,
                                                          const float* __restrict__ scale, float4* __restrict__ scaled,
                                                          uint2* __restrict__ shi, uint2* __restrict__ slo,
                                                          int64_t groups, int nch, int rows, int cols4, int reverse) {
  constexpr int kB = 8;
  const int64_t rc4 = (int64_t)rows * cols4;
  const int64_t e = blockIdx.x * 256ll + threadIdx.x;
  if (e >= groups * rc4) return;
  const int64_t grp = e / rc4, w = e % rc4;
  const int r = (int)(w / cols4);
  float4* xp = x + grp * nch * rc4 + w;
  float4* op = scaled ? scaled + grp * nch * rc4 + w : nullptr;
  const float* dp = decay ? decay + grp * nch * rows + r : nullptr;
  const float* sp = scale ? scale + grp * nch * rows + r : nullptr;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int it0 = 0; it0 < nch; it0 += kB) {
    float4 y[kB];
    float dc[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int it = it0 + u;
      const int kc = reverse ? nch - 1 - it : it;
      y[u] = it < nch ? xp[kc * rc4] : make_float4(0.f, 0.f, 0.f, 0.f);
      dc[u] = (it < nch && dp) ? dp[(int64_t)kc * rows] : 1.f;
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int it = it0 + u;
      if (it < nch) {
        const int kc = reverse ? nch - 1 - it : it;
        xp[kc * rc4] = s;
        const float f = sp ? sp[(int64_t)kc * rows] : 1.f;
        const float4 fs = make_float4(f * s.x, f * s.y, f * s.z, f * s.w);
        if (op) op[kc * rc4] = fs;
        if (shi) {  // 4 bf16 high parts (and low parts) in 8 bytes each
          const int64_t o = grp * nch * rc4 + w + kc * rc4;
          const __nv_bfloat162 h01 = __floats2bfloat162_rn(fs.x, fs.y), h23 = __floats2bfloat162_rn(fs.z, fs.w);
          shi[o] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
          if (slo) {
            const float2 b01 = __bfloat1622float2(h01), b23 = __bfloat1622float2(h23);
            const __nv_bfloat162 l01 = __floats2bfloat162_rn(fs.x - b01.x, fs.y - b01.y);
            const __nv_bfloat162 l23 = __floats2bfloat162_rn(fs.z - b23.x, fs.w - b23.y);
            slo[o] = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
          }
        }
        s = make_float4(fmaf(dc[u], s.x, y[u].x), fmaf(dc[u], s.y, y[u].y), fmaf(dc[u], s.z, y[u].z),
                        fmaf(dc[u], s.w, y[u].w));
      }
    }
  }
}

// Row mode of the chunk-state scan (tensor-core backward): one warp per (group, row),
// lane l owning the float4 columns l, l + 32, ... (NV of them).  Per chunk in order (or
// reversed): the exclusive state s is written as the bf16 high / low split of scale * s
// (and to x_out unless skipped), with dot the inner product of s with the next chunk's
// state read back from the state scan's split copy (divided by its scale), reduced over
// the warp; then s = decay * s + x_in[chunk].  The next chunk's increments are loaded
// while the current one is written.
template <int NV>
__global__ void __launch_bounds__(256) chunk_scan_rows_kernel(
    const float* __restrict__ x_in, float* __restrict__ x_out, const float* __restrict__ decay,
    const float* __restrict__ scale, uint2* __restrict__ shi, uint2* __restrict__ slo, const uint2* __restrict__ dhi,
    const uint2* __restrict__ dlo, const float* __restrict__ dscale, float* __restrict__ dout, int64_t groups, int nch,
    int rows, int cols, int reverse) {
  const int lane = threadIdx.x & 31;
  const int64_t wr = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (wr >= groups * rows) return;
  const int64_t grp = wr / rows;
  const int r = (int)(wr % rows);
  const int cols4 = cols >> 2;
  const int64_t rc4 = (int64_t)rows * cols4;                 // float4s per chunk
  const int64_t base4 = grp * nch * rc4 + (int64_t)r * cols4;  // (grp, chunk 0, r, 0)
  const int64_t vbase = grp * nch * rows + r;
  const float4* xin4 = reinterpret_cast<const float4*>(x_in);
  float4* xout4 = reinterpret_cast<float4*>(x_out);
  float4 s[NV], y[NV];
  auto load = [&](int it, float4 (&dst)[NV]) {
    const int kc = reverse ? nch - 1 - it : it;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c4 = lane + 32 * v;
      dst[v] = (it < nch && c4 < cols4) ? xin4[base4 + kc * rc4 + c4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
#pragma unroll
  for (int v = 0; v < NV; ++v) s[v] = make_float4(0.f, 0.f, 0.f, 0.f);
  load(0, y);
  for (int it = 0; it < nch; ++it) {
    const int kc = reverse ? nch - 1 - it : it;
    float4 yn[NV];
    load(it + 1, yn);
    const float dc = decay ? decay[vbase + (int64_t)kc * rows] : 1.f;
    const float f = scale ? scale[vbase + (int64_t)kc * rows] : 1.f;
    const int64_t o4 = base4 + kc * rc4;
    const int kn = kc + 1;
    const bool dot = dout && kn < nch;
    const float inv = (dot && dscale) ? 1.f / dscale[vbase + (int64_t)kn * rows] : 1.f;
    float part = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c4 = lane + 32 * v;
      if (c4 >= cols4) continue;
      const float4 z = s[v];
      if (xout4) xout4[o4 + c4] = z;
      const float4 fs = make_float4(f * z.x, f * z.y, f * z.z, f * z.w);
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(fs.x, fs.y), h23 = __floats2bfloat162_rn(fs.z, fs.w);
      shi[o4 + c4] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
      if (slo) {
        const float2 b01 = __bfloat1622float2(h01), b23 = __bfloat1622float2(h23);
        const __nv_bfloat162 l01 = __floats2bfloat162_rn(fs.x - b01.x, fs.y - b01.y);
        const __nv_bfloat162 l23 = __floats2bfloat162_rn(fs.z - b23.x, fs.w - b23.y);
        slo[o4 + c4] = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
      }
      if (dot) {  // the next chunk's state: (hi + lo) / its scale
        const int64_t n4 = base4 + kn * rc4 + c4;
        const uint2 hh = dhi[n4];
        float2 a01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hh.x));
        float2 a23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hh.y));
        if (dlo) {
          const uint2 ll = dlo[n4];
          const float2 c01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ll.x));
          const float2 c23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ll.y));
          a01.x += c01.x; a01.y += c01.y; a23.x += c23.x; a23.y += c23.y;
        }
        part = fmaf(z.x, a01.x, fmaf(z.y, a01.y, fmaf(z.z, a23.x, fmaf(z.w, a23.y, part))));
      }
    }
    if (dout) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      if (lane == 0) dout[vbase + (int64_t)kc * rows] = dot ? part * inv : 0.f;
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      s[v] = make_float4(fmaf(dc, s[v].x, y[v].x), fmaf(dc, s[v].y, y[v].y), fmaf(dc, s[v].z, y[v].z),
                         fmaf(dc, s[v].w, y[v].w));
      y[v] = yn[v];
    }
  }
}

// Output-side gradients of one chunk row t (one warp per row): from the chunk
// outputs [num | den] (width w, fp32) and dh, with D = max(den, 1),
//   dnum = dh / D,  dden = -[den >= 1] (dnum . num) / D     (normalize)
//   dnum = dh,      dden = 0                                 (no normalizer)
// written as [dnum | dden | 0 ...] (width w); rows t >= seqlen are zero.
template <typename T>
__global__ void __launch_bounds__(256) normalizer_kernel(const float* __restrict__ numa, const T* __restrict__ dh,
                                                         int64_t sb, int64_t sh, int64_t st, int heads, int seqlen,
                                                         int lp, int dv, int w, int normalize, int64_t rows,
                                                         float* __restrict__ dna, __nv_bfloat16* __restrict__ dhi,
                                                         __nv_bfloat16* __restrict__ dlo) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int t = (int)(row % lp);
  const int64_t bh = row / lp;
  const int b = (int)(bh / heads), h = (int)(bh % heads);
  const float* nrow = numa + row * w;
  // one output element: fp32 and / or the bf16 high / low parts
  auto put = [&](int e, float x) {
    if (dna) dna[row * w + e] = x;
    if (dhi) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(x);
      dhi[row * w + e] = hi;
      if (dlo) dlo[row * w + e] = __float2bfloat16_rn(x - __bfloat162float(hi));
    }
  };
  if (t >= seqlen) {
    for (int e = lane; e < w; e += 32) put(e, 0.f);
    return;
  }
  const T* drow = dh + b * sb + h * sh + (int64_t)t * st;
  const float den = normalize ? nrow[dv] : 1.f;
  const float inv = 1.f / fmaxf(den, 1.f);
  float part = 0.f;
  for (int e = lane; e < dv; e += 32) {
    const float g = to_f32<T>(drow[e]) * inv;
    put(e, g);
    if (normalize) part = fmaf(g, nrow[e], part);  // (outputs is unread, and may be NULL, without it)
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  for (int e = dv + lane; e < w; e += 32) put(e, (e == dv && normalize && den >= 1.f) ? -part * inv : 0.f);
}

// out[g, k, r] = sum_c adj[g, k, r, c] * state[g, k + 1, r, c]  (0 for the last
// chunk): one warp per (g, k, r) row, 16-byte loads when VEC.
template <bool VEC>
__global__ void __launch_bounds__(256) chunk_dot_kernel(const float* __restrict__ adj, const float* __restrict__ state,
                                                        int64_t groups, int nch, int rows, int cols,
                                                        float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (row >= groups * nch * rows) return;
  const int r = (int)(row % rows);
  const int64_t gk = row / rows;
  const int kc = (int)(gk % nch);
  const int64_t grp = gk / nch;
  if (kc == nch - 1) {
    if (lane == 0) out[row] = 0.f;
    return;
  }
  const float* a = adj + row * cols;
  const float* x = state + ((grp * nch + kc + 1) * rows + r) * (int64_t)cols;
  float acc = 0.f;
  if (VEC) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int c = lane; c < cols / 4; c += 32) {
      const float4 u = a4[c], v = x4[c];
      acc = fmaf(u.x, v.x, fmaf(u.y, v.y, fmaf(u.z, v.z, fmaf(u.w, v.w, acc))));
    }
  } else {
    for (int c = lane; c < cols; c += 32) acc = fmaf(a[c], x[c], acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = acc;
}

static unsigned grid_each(int64_t n) { return (unsigned)((n + 255) / 256); }

static hxm_status fill(const hxm_mlstm_bwd_args* a, Params& p, const char* who) {
  HXM_REQUIRE(a != nullptr, "%s: args is NULL", who);
  HXM_REQUIRE(a->struct_size == sizeof(hxm_mlstm_bwd_args), "%s: struct_size %zu != %zu", who, a->struct_size,
              sizeof(hxm_mlstm_bwd_args));
  HXM_REQUIRE(a->batch >= 1 && a->heads >= 1 && a->seqlen >= 0 && a->dqk >= 1,
              "%s: bad sizes batch=%d heads=%d seqlen=%d dqk=%d", who, a->batch, a->heads, a->seqlen, a->dqk);
  HXM_REQUIRE(a->chunk >= 1 && a->chunk <= 1024, "%s: chunk must be in [1, 1024] (got %d)", who, a->chunk);
  HXM_REQUIRE(a->gate_mode == 0 || a->gate_mode == 1, "%s: gate_mode must be 0 or 1", who);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "%s: io_dtype must be f32 or bf16", who);
  p.batch = a->batch; p.heads = a->heads; p.seqlen = a->seqlen; p.dqk = a->dqk; p.chunk = a->chunk;
  p.nch = (a->seqlen + a->chunk - 1) / a->chunk;
  p.gate_mode = a->gate_mode;
  p.q = a->q; p.k = a->k; p.log_i = a->log_i; p.log_f = a->log_f;
  for (int i = 0; i < 3; ++i) {
    p.sq[i] = a->q_stride[i]; p.sk[i] = a->k_stride[i]; p.si[i] = a->i_stride[i]; p.sf[i] = a->f_stride[i];
  }
  p.qs = a->q_scaled; p.ks = a->k_scaled; p.rho = a->rho; p.erho = a->e_rho; p.eg = a->e_g;
  p.qd = a->q_decayed; p.kd = a->k_decayed;
  p.planes = static_cast<__nv_bfloat16*>(a->split_planes);
  p.plane = (int64_t)p.batch * p.heads * p.nch * p.chunk * p.dqk;
  p.dqs = a->dq_scaled; p.dks = a->dk_scaled; p.dg = a->chunk_dg;
  p.dq = a->dq; p.dk = a->dk; p.dli = a->dlog_i; p.dlf = a->dlog_f; p.di = a->d_i;
  HXM_REQUIRE(p.log_i && p.log_f && ((p.qs && p.ks) || p.planes) && p.rho, "%s: NULL gate or chunk-operand pointer",
              who);
  return HXM_OK;
}

}  // namespace mlstm_bwd
}  // namespace hxm

extern "C" hxm_status hxm_mlstm_bwd_prepare(const hxm_mlstm_bwd_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  mlstm_bwd::Params p{};
  hxm_status s = mlstm_bwd::fill(a, p, "hxm_mlstm_bwd_prepare");
  if (s != HXM_OK) return s;
  HXM_REQUIRE(p.q && p.k && p.erho && p.eg, "hxm_mlstm_bwd_prepare: NULL q, k, e_rho or e_g");
  if (p.nch == 0) return HXM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.batch * p.heads * p.nch), (unsigned)((p.dqk + 127) / 128));
  if (a->io_dtype == HXM_F32) mlstm_bwd::prepare_kernel<float><<<grid, 128, 0, st>>>(p);
  else mlstm_bwd::prepare_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(p);
  return check_launch("hxm_mlstm_bwd_prepare");
}

extern "C" hxm_status hxm_mlstm_bwd_finalize(const hxm_mlstm_bwd_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  mlstm_bwd::Params p{};
  hxm_status s = mlstm_bwd::fill(a, p, "hxm_mlstm_bwd_finalize");
  if (s != HXM_OK) return s;
  HXM_REQUIRE(p.dqs && p.dks && p.dg && p.dq && p.dk && p.dli && p.dlf,
              "hxm_mlstm_bwd_finalize: NULL gradient or chunk_dg pointer");
  if (p.nch == 0) return HXM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(p.batch * p.heads * p.nch), (unsigned)((p.dqk + 127) / 128));
  HXM_REQUIRE(p.k || !p.di, "hxm_mlstm_bwd_finalize: d_i needs k");
  if (a->io_dtype == HXM_F32) mlstm_bwd::finalize_kernel<float><<<grid, 128, 0, st>>>(p);
  else mlstm_bwd::finalize_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(p);
  return check_launch("hxm_mlstm_bwd_finalize");
}

extern "C" hxm_status hxm_chunk_state_scan(const hxm_chunk_scan_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_chunk_state_scan: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_chunk_scan_args), "hxm_chunk_state_scan: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_chunk_scan_args));
  HXM_REQUIRE(a->groups >= 0 && a->nchunks >= 0 && a->rows >= 1 && a->cols >= 1,
              "hxm_chunk_state_scan: bad sizes groups=%lld nchunks=%d rows=%d cols=%d", (long long)a->groups,
              a->nchunks, a->rows, a->cols);
  if (a->groups == 0 || a->nchunks == 0) return HXM_OK;
  HXM_REQUIRE(a->x != nullptr, "hxm_chunk_state_scan: x is NULL");
  HXM_REQUIRE(!a->scaled || a->scale, "hxm_chunk_state_scan: scaled output needs scale");
  HXM_REQUIRE(!a->scaled_lo || a->scaled_hi, "hxm_chunk_state_scan: scaled_lo needs scaled_hi");
  const int64_t n = a->groups * a->rows * (int64_t)a->cols;
  HXM_REQUIRE(n / 256 < (int64_t)0x7fffffff, "hxm_chunk_state_scan: too many elements (%lld)", (long long)n);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool row_ok = a->scaled_hi && !a->scaled && a->cols % 4 == 0 && a->cols <= 640 &&
                      reinterpret_cast<uintptr_t>(a->x) % 16 == 0 && reinterpret_cast<uintptr_t>(a->scaled_hi) % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(a->scaled_lo) % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(a->dot_hi) % 8 == 0 && reinterpret_cast<uintptr_t>(a->dot_lo) % 8 == 0;
  HXM_REQUIRE_SUPPORTED(row_ok || (!a->dot_out && !a->skip_state),
                        "hxm_chunk_state_scan: dot_out / skip_state need the row mode (scaled_hi without scaled, "
                        "cols %% 4 == 0 and <= 640, aligned pointers)");
  HXM_REQUIRE(!a->dot_out || a->dot_hi, "hxm_chunk_state_scan: dot_out needs dot_hi");
  if (row_ok) {
    const int nv = (a->cols / 4 + 31) / 32;
    const unsigned grid = (unsigned)((a->groups * a->rows + 7) / 8);
    float* xo = a->skip_state ? nullptr : a->x;
    auto* hi = static_cast<uint2*>(a->scaled_hi);
    auto* lo = static_cast<uint2*>(a->scaled_lo);
    auto* dh = static_cast<const uint2*>(a->dot_hi);
    auto* dl = static_cast<const uint2*>(a->dot_lo);
#define HXM_ROWS(NV)                                                                                           \
  mlstm_bwd::chunk_scan_rows_kernel<NV><<<grid, 256, 0, st>>>(a->x, xo, a->decay, a->scale, hi, lo, dh, dl,    \
                                                              a->dot_scale, a->dot_out, a->groups, a->nchunks, \
                                                              a->rows, a->cols, a->reverse ? 1 : 0)
    switch (nv) {
      case 1: HXM_ROWS(1); break;
      case 2: HXM_ROWS(2); break;
      case 3: HXM_ROWS(3); break;
      case 4: HXM_ROWS(4); break;
      default: HXM_ROWS(5); break;
    }
#undef HXM_ROWS
    return check_launch("hxm_chunk_state_scan (rows)");
  }
  if (a->cols % 4 == 0 && reinterpret_cast<uintptr_t>(a->x) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(a->scaled) % 16 == 0 && reinterpret_cast<uintptr_t>(a->scaled_hi) % 8 == 0 &&
      reinterpret_cast<uintptr_t>(a->scaled_lo) % 8 == 0)
    mlstm_bwd::chunk_scan4_kernel<<<mlstm_bwd::grid_each(n / 4), 256, 0, st>>>(
        reinterpret_cast<float4*>(a->x), a->decay, a->scale, reinterpret_cast<float4*>(a->scaled),
        static_cast<uint2*>(a->scaled_hi), static_cast<uint2*>(a->scaled_lo), a->groups, a->nchunks, a->rows,
        a->cols / 4, a->reverse ? 1 : 0);
  else
    mlstm_bwd::chunk_scan_kernel<<<mlstm_bwd::grid_each(n), 256, 0, st>>>(
        a->x, a->decay, a->scale, a->scaled, static_cast<__nv_bfloat16*>(a->scaled_hi),
        static_cast<__nv_bfloat16*>(a->scaled_lo), a->groups, a->nchunks, a->rows, a->cols, a->reverse ? 1 : 0);
  return check_launch("hxm_chunk_state_scan");
}

extern "C" hxm_status hxm_mlstm_bwd_normalizer(const hxm_mlstm_bwd_norm_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_mlstm_bwd_normalizer: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_mlstm_bwd_norm_args), "hxm_mlstm_bwd_normalizer: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_mlstm_bwd_norm_args));
  HXM_REQUIRE(a->batch >= 0 && a->heads >= 1 && a->seqlen >= 0 && a->padded_len >= a->seqlen && a->dv >= 1 &&
                  a->width >= a->dv + (a->normalize ? 1 : 0),
              "hxm_mlstm_bwd_normalizer: bad sizes batch=%d heads=%d seqlen=%d padded_len=%d dv=%d width=%d",
              a->batch, a->heads, a->seqlen, a->padded_len, a->dv, a->width);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "hxm_mlstm_bwd_normalizer: io_dtype must be f32 or bf16");
  const int64_t rows = (int64_t)a->batch * a->heads * a->padded_len;
  if (rows == 0) return HXM_OK;
  HXM_REQUIRE((a->out || a->out_hi) && a->dh && (a->outputs || !a->normalize), "hxm_mlstm_bwd_normalizer: NULL pointer");
  HXM_REQUIRE(!a->out_lo || a->out_hi, "hxm_mlstm_bwd_normalizer: out_lo needs out_hi");
  const unsigned grid = (unsigned)((rows + 7) / 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* numa = a->outputs;  // unread without the normalizer
  auto* ohi = static_cast<__nv_bfloat16*>(a->out_hi);
  auto* olo = static_cast<__nv_bfloat16*>(a->out_lo);
  if (a->io_dtype == HXM_F32)
    mlstm_bwd::normalizer_kernel<float><<<grid, 256, 0, st>>>(
        numa, static_cast<const float*>(a->dh), a->dh_stride[0], a->dh_stride[1], a->dh_stride[2], a->heads,
        a->seqlen, a->padded_len, a->dv, a->width, a->normalize ? 1 : 0, rows, a->out, ohi, olo);
  else
    mlstm_bwd::normalizer_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        numa, static_cast<const __nv_bfloat16*>(a->dh), a->dh_stride[0], a->dh_stride[1], a->dh_stride[2], a->heads,
        a->seqlen, a->padded_len, a->dv, a->width, a->normalize ? 1 : 0, rows, a->out, ohi, olo);
  return check_launch("hxm_mlstm_bwd_normalizer");
}

extern "C" hxm_status hxm_chunk_state_dot(const hxm_chunk_dot_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_chunk_state_dot: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_chunk_dot_args), "hxm_chunk_state_dot: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_chunk_dot_args));
  HXM_REQUIRE(a->groups >= 0 && a->nchunks >= 0 && a->rows >= 1 && a->cols >= 1,
              "hxm_chunk_state_dot: bad sizes groups=%lld nchunks=%d rows=%d cols=%d", (long long)a->groups,
              a->nchunks, a->rows, a->cols);
  const int64_t nrows = a->groups * a->nchunks * (int64_t)a->rows;
  if (nrows == 0) return HXM_OK;
  HXM_REQUIRE(a->adj && a->state && a->out, "hxm_chunk_state_dot: NULL pointer");
  HXM_REQUIRE((nrows + 7) / 8 < (int64_t)0x7fffffff, "hxm_chunk_state_dot: too many rows (%lld)", (long long)nrows);
  const unsigned grid = (unsigned)((nrows + 7) / 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = a->cols % 4 == 0 && reinterpret_cast<uintptr_t>(a->adj) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a->state) % 16 == 0;
  if (vec)
    mlstm_bwd::chunk_dot_kernel<true><<<grid, 256, 0, st>>>(a->adj, a->state, a->groups, a->nchunks, a->rows, a->cols,
                                                            a->out);
  else
    mlstm_bwd::chunk_dot_kernel<false><<<grid, 256, 0, st>>>(a->adj, a->state, a->groups, a->nchunks, a->rows,
                                                             a->cols, a->out);
  return check_launch("hxm_chunk_state_dot");
}
