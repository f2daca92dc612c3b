// scan_bwd.cu — selective-scan backward (Euler) for sm_100a.
//
// Replaces the backward of SelectiveScanFunction
// (hybrid_xmamba/kernels/selective_scan/scan_interface.py:62-100), which
// re-runs the reference loop under autograd.  Forward per channel d:
//   delta_t = softplus(raw_t + bias) (or raw_t + bias, or raw_t)
//   a_t[n]  = exp(delta_t A[n]),  h_t = a_t h_{t-1} + delta_t B_t u_t
//   y_t     = C_t . h_t + D u_t,  out_t = y_t * gate(z_t)
// Backward, reverse in time, with dh_t = dy_t C_t + a_{t+1} dh_{t+1}:
//   dC_t += dy_t h_t,  dB_t += dh_t delta_t u_t,  dA += dh_t h_{t-1} a_t delta_t,
//   ddelta_t = sum_n dh_t (h_{t-1} a_t A + B_t u_t),
//   du_t = dy_t D + delta_t dh_t . B_t,  dD += dy_t u_t.
// One thread per (batch row, channel), 16 fp32 states in registers; the B, C
// rows of each 16-step chunk are staged in shared memory for the whole CTA.
// A first pass recomputes the forward and stores h every 16 steps in the
// workspace;
// the reverse pass reloads each checkpoint, recomputes the chunk's h_{t-1}
// into shared memory and walks it backwards.  dB, dC are sums over channels:
// a warp reduce-scatter leaves lane l with the warp's sum of value l, one
// atomicAdd per warp.  dA, dD, dbias sum over time in registers and over the
// batch with atomics.
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace scanbwd {

constexpr int CH = 64;   // channels per CTA (one per thread)
constexpr int kT = 16;   // checkpoint interval
constexpr int NS = 16;   // max dstate

struct Params {
  int batch, seqlen, dim, dstate;
  const void *u, *dt, *B, *C, *z, *dout;
  int64_t su[3], sdt[3], sB[3], sC[3], sz[3], sdo[3];
  const float *A, *D, *bias, *h0;
  int64_t sA[2];
  float *du, *ddt, *dz, *dA, *dB, *dC, *dD, *dbias, *dh0;
  float* ckpt;
};

HXM_DEV float sigmoid_acc(float x) { return 1.f / (1.f + expf(-x)); }

template <typename T>
HXM_DEV float ld(const void* base, const int64_t* s, int b, int t, int c) {
  return to_f32<T>(static_cast<const T*>(base)[b * s[0] + (int64_t)t * s[1] + (int64_t)c * s[2]]);
}

template <typename T, int ZMODE, bool SP>
__global__ void __launch_bounds__(CH) scan_bwd_kernel(const Params p) {
  extern __shared__ float hs[];  // [kT][NS][CH]: h_{t-1} of the chunk, then [3][kT][CH]
  float* sdl = hs + kT * NS * CH;   // delta_t of the chunk (per channel)
  float* suv = sdl + kT * CH;       // u_t
  float* ssg = suv + kT * CH;       // d delta / d raw (softplus' derivative, or 1)
  const int tid = threadIdx.x, lane = tid & 31;
  const int b = blockIdx.y;
  const int d = blockIdx.x * CH + tid;
  const bool dvalid = d < p.dim;
  const int dc = dvalid ? d : 0;
  const int N = p.dstate;
  const int nck = (p.seqlen + kT - 1) / kT;

  // a[n] = A[d, n]; a2[n] = A[d, n] log2(e): exp(delta A) = 2^(delta a2) on the MUFU unit
  // (relative error ~2e-7, the forward kernel's exponential)
  float a[NS], a2[NS];
#pragma unroll
  for (int n = 0; n < NS; ++n) {
    a[n] = n < N ? p.A[(int64_t)dc * p.sA[0] + (int64_t)n * p.sA[1]] : 0.f;
    a2[n] = a[n] * kLog2e;
  }
  const float Dd = p.D ? p.D[dc] : 0.f;
  const float bias = p.bias ? p.bias[dc] : 0.f;
  float* ck = p.ckpt + ((int64_t)b * p.dim + dc) * nck * NS;

  auto delta_of = [&](int t, float& raw) {
    raw = ld<T>(p.dt, p.sdt, b, t, dc) + bias;
    return SP ? softplus<false>(raw) : raw;
  };

  // B, C of one kT-step chunk staged in shared memory (fp32, zero past the
  // sequence / dstate): every thread of the CTA reads the same rows
  __shared__ float sbc[2][kT][NS];
  auto stage = [&](int k, int nw) {
    const int t0 = k * kT;
    for (int e = tid; e < nw * kT * NS; e += CH) {
      const int w = e / (kT * NS), i = (e / NS) % kT, n = e % NS;
      const int t = t0 + i;
      float v = 0.f;
      if (t < p.seqlen && n < N) v = w ? ld<T>(p.C, p.sC, b, t, n) : ld<T>(p.B, p.sB, b, t, n);
      sbc[w][i][n] = v;
    }
  };

  // ---- pass 1: forward recompute, checkpoints every kT steps -----------------
  float h[NS];
#pragma unroll
  for (int n = 0; n < NS; ++n) h[n] = (p.h0 && n < N) ? p.h0[((int64_t)b * p.dim + dc) * N + n] : 0.f;
  for (int k = 0; k < nck; ++k) {
    const int t0 = k * kT, tn = min(kT, p.seqlen - t0);
    __syncthreads();  // the previous chunk's rows are consumed
    stage(k, 1);
    __syncthreads();
    if (dvalid) {
#pragma unroll
      for (int n = 0; n < NS; ++n) ck[k * NS + n] = h[n];
    }
    for (int i = 0; i < tn; ++i) {
      float raw;
      const float dl = delta_of(t0 + i, raw);
      const float du = dl * ld<T>(p.u, p.su, b, t0 + i, dc);
#pragma unroll
      for (int n = 0; n < NS; ++n)
        if (n < N) h[n] = fmaf(ex2_approx(dl * a2[n]), h[n], du * sbc[0][i][n]);
    }
  }

  // ---- pass 2: reverse ------------------------------------------------------
  float dh[NS], dAacc[NS];
#pragma unroll
  for (int n = 0; n < NS; ++n) dh[n] = dAacc[n] = 0.f;
  float dDacc = 0.f, dbacc = 0.f;
  for (int k = nck - 1; k >= 0; --k) {
    const int t0 = k * kT, tn = min(kT, p.seqlen - t0);
    __syncthreads();
    stage(k, 2);
    __syncthreads();
#pragma unroll
    for (int n = 0; n < NS; ++n) h[n] = dvalid ? ck[k * NS + n] : 0.f;
    for (int i = 0; i < tn; ++i) {
      const int t = t0 + i;
#pragma unroll
      for (int n = 0; n < NS; ++n) hs[(i * NS + n) * CH + tid] = h[n];
      float raw;
      const float dl = delta_of(t, raw);
      const float uv = ld<T>(p.u, p.su, b, t, dc);
      const float du = dl * uv;
      sdl[i * CH + tid] = dl;
      suv[i * CH + tid] = uv;
      ssg[i * CH + tid] = SP ? (raw > 20.f ? 1.f : sigmoid_acc(raw)) : 1.f;
#pragma unroll
      for (int n = 0; n < NS; ++n)
        if (n < N) h[n] = fmaf(ex2_approx(dl * a2[n]), h[n], du * sbc[0][i][n]);
    }
    for (int i = tn - 1; i >= 0; --i) {
      const int t = t0 + i;
      const float dl = sdl[i * CH + tid];
      const float u = suv[i * CH + tid];
      const float go = dvalid ? ld<T>(p.dout, p.sdo, b, t, dc) : 0.f;
      float Bv[NS], Cv[NS], hp[NS], at[NS];
      float y = Dd * u;
#pragma unroll
      for (int n = 0; n < NS; ++n) {
        Bv[n] = sbc[0][i][n];
        Cv[n] = sbc[1][i][n];
        hp[n] = hs[(i * NS + n) * CH + tid];
        at[n] = n < N ? ex2_approx(dl * a2[n]) : 0.f;
        y = fmaf(Cv[n], fmaf(at[n], hp[n], dl * Bv[n] * u), y);
      }
      float dy = go, dzv = 0.f;
      if (ZMODE == 1) {
        const float zv = ld<T>(p.z, p.sz, b, t, dc);
        dy = go * zv;
        dzv = go * y;
      } else if (ZMODE == 2) {
        const float zv = ld<T>(p.z, p.sz, b, t, dc);
        const float s = sigmoid_acc(zv);
        dy = go * zv * s;
        dzv = go * y * s * (1.f + zv * (1.f - s));
      }
      dDacc = fmaf(dy, u, dDacc);
      float duv = dy * Dd, ddl = 0.f;
      float red[2 * NS];  // [dB_t partial | dC_t partial]
#pragma unroll
      for (int n = 0; n < NS; ++n) {
        const float ht = fmaf(at[n], hp[n], dl * Bv[n] * u);
        dh[n] = fmaf(dy, Cv[n], dh[n]);
        red[NS + n] = dvalid ? dy * ht : 0.f;
        const float da = dh[n] * hp[n];
        ddl = fmaf(da * at[n], a[n], ddl);
        ddl = fmaf(dh[n], Bv[n] * u, ddl);
        dAacc[n] = fmaf(da * at[n], dl, dAacc[n]);
        red[n] = dvalid ? dh[n] * dl * u : 0.f;
        duv = fmaf(dh[n] * dl, Bv[n], duv);
        dh[n] *= at[n];
      }
      const float draw = ddl * ssg[i * CH + tid];
      dbacc += draw;
      if (dvalid) {
        const int64_t o = ((int64_t)b * p.seqlen + t) * p.dim + d;
        if (p.du) p.du[o] = duv;
        if (p.ddt) p.ddt[o] = draw;
        if (ZMODE != 0 && p.dz) p.dz[o] = dzv;
      }
      // warp reduce-scatter of the 32 partials: lane l ends with the warp sum of red[l]
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
        for (int j = 0; j < off; ++j) {
          const bool up = lane & off;
          const float send = up ? red[j] : red[j + off];
          const float keep = up ? red[j + off] : red[j];
          red[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int n = lane & (NS - 1);
      if (n < N) {
        float* dst = lane < NS ? p.dB : p.dC;
        if (dst) atomicAdd(dst + ((int64_t)b * p.seqlen + t) * N + n, red[0]);
      }
    }
  }
  if (dvalid) {
#pragma unroll
    for (int n = 0; n < NS; ++n) {
      if (n < N) {
        if (p.dA) atomicAdd(p.dA + (int64_t)d * N + n, dAacc[n]);
        if (p.dh0) p.dh0[((int64_t)b * p.dim + d) * N + n] = dh[n];
      }
    }
    if (p.dD) atomicAdd(p.dD + d, dDacc);
    if (p.dbias) atomicAdd(p.dbias + d, dbacc);
  }
}

template <typename T, int ZMODE, bool SP>
hxm_status launch(const Params& p, cudaStream_t st) {
  const size_t smem = sizeof(float) * kT * (NS + 3) * CH;
  auto kern = scan_bwd_kernel<T, ZMODE, SP>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dim + CH - 1) / CH, p.batch);
  kern<<<grid, CH, smem, st>>>(p);
  return check_launch("hxm_selective_scan_bwd");
}

template <typename T>
hxm_status dispatch(const Params& p, int zmode, bool sp, cudaStream_t st) {
  if (sp) {
    if (zmode == 2) return launch<T, 2, true>(p, st);
    if (zmode == 1) return launch<T, 1, true>(p, st);
    return launch<T, 0, true>(p, st);
  }
  if (zmode == 2) return launch<T, 2, false>(p, st);
  if (zmode == 1) return launch<T, 1, false>(p, st);
  return launch<T, 0, false>(p, st);
}

static size_t workspace(const hxm_scan_args& f) {
  const size_t nck = ((size_t)f.seqlen + kT - 1) / kT;
  return sizeof(float) * (size_t)f.batch * f.dim * nck * NS;
}

static hxm_status check(const hxm_scan_bwd_args* a) {
  HXM_REQUIRE(a != nullptr, "hxm_selective_scan_bwd: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_scan_bwd_args) && a->fwd.struct_size == sizeof(hxm_scan_args),
              "hxm_selective_scan_bwd: struct_size mismatch");
  const hxm_scan_args& f = a->fwd;
  HXM_REQUIRE(f.batch >= 0 && f.seqlen >= 0 && f.dim >= 0 && f.dstate >= 1, "hxm_selective_scan_bwd: bad dims");
  HXM_REQUIRE_SUPPORTED(f.dstate <= NS, "hxm_selective_scan_bwd: dstate %d > %d unsupported", f.dstate, NS);
  HXM_REQUIRE_SUPPORTED(f.discretization == 0, "hxm_selective_scan_bwd: only the Euler discretization");
  HXM_REQUIRE(f.io_dtype == HXM_F32 || f.io_dtype == HXM_BF16, "hxm_selective_scan_bwd: io_dtype must be f32 or bf16");
  HXM_REQUIRE(f.z_mode >= 0 && f.z_mode <= 2 && (f.z_mode == 0 || f.z), "hxm_selective_scan_bwd: bad z_mode / z");
  HXM_REQUIRE((int64_t)f.batch <= 65535, "hxm_selective_scan_bwd: batch > 65535");
  return HXM_OK;
}

}  // namespace scanbwd
}  // namespace hxm

extern "C" size_t hxm_selective_scan_bwd_workspace_size(const hxm_scan_bwd_args* a) {
  if (hxm::scanbwd::check(a) != HXM_OK) return 0;
  return hxm::scanbwd::workspace(a->fwd);
}

extern "C" hxm_status hxm_selective_scan_bwd(const hxm_scan_bwd_args* a, void* stream_) {
  using namespace hxm;
  clear_error();
  hxm_status s = scanbwd::check(a);
  if (s != HXM_OK) return s;
  const hxm_scan_args& f = a->fwd;
  cudaStream_t st = static_cast<cudaStream_t>(stream_);
  // the sums over time / batch / channels accumulate with atomics: start from zero
  auto zero = [&](float* ptr, size_t n) -> hxm_status {
    if (ptr && n) HXM_CUDA_TRY(cudaMemsetAsync(ptr, 0, n * sizeof(float), st));
    return HXM_OK;
  };
  const size_t bld = (size_t)f.batch * f.seqlen * f.dim, bln = (size_t)f.batch * f.seqlen * f.dstate;
  if ((s = zero(a->dA, (size_t)f.dim * f.dstate)) != HXM_OK) return s;
  if ((s = zero(a->dB, bln)) != HXM_OK) return s;
  if ((s = zero(a->dC, bln)) != HXM_OK) return s;
  if ((s = zero(a->dD, f.dim)) != HXM_OK) return s;
  if ((s = zero(a->ddelta_bias, f.dim)) != HXM_OK) return s;
  if (f.batch == 0 || f.dim == 0) return HXM_OK;
  if (f.seqlen == 0) {
    if ((s = zero(a->du, bld)) != HXM_OK) return s;
    if (a->dh0) HXM_CUDA_TRY(cudaMemsetAsync(a->dh0, 0, sizeof(float) * f.batch * f.dim * f.dstate, st));
    return HXM_OK;
  }
  HXM_REQUIRE(f.u && f.delta && f.A && f.B && f.C && a->dout, "hxm_selective_scan_bwd: NULL tensor pointer");
  const size_t need = scanbwd::workspace(f);
  HXM_REQUIRE(a->workspace && a->workspace_bytes >= need, "hxm_selective_scan_bwd: workspace of %zu bytes required",
              need);
  scanbwd::Params p{};
  p.batch = f.batch; p.seqlen = f.seqlen; p.dim = f.dim; p.dstate = f.dstate;
  p.u = f.u; p.dt = f.delta; p.B = f.B; p.C = f.C; p.z = f.z; p.dout = a->dout;
  for (int i = 0; i < 3; ++i) {
    p.su[i] = f.u_stride[i]; p.sdt[i] = f.delta_stride[i]; p.sB[i] = f.B_stride[i]; p.sC[i] = f.C_stride[i];
    p.sz[i] = f.z_stride[i]; p.sdo[i] = a->dout_stride[i];
  }
  p.A = f.A; p.sA[0] = f.A_stride[0]; p.sA[1] = f.A_stride[1];
  p.D = f.D; p.bias = f.delta_bias; p.h0 = f.h0;
  p.du = a->du; p.ddt = a->ddelta; p.dz = a->dz; p.dA = a->dA; p.dB = a->dB; p.dC = a->dC; p.dD = a->dD;
  p.dbias = a->ddelta_bias; p.dh0 = a->dh0;
  p.ckpt = static_cast<float*>(a->workspace);
  const int zm = f.z ? f.z_mode : 0;
  return f.io_dtype == HXM_F32 ? scanbwd::dispatch<float>(p, zm, f.delta_softplus != 0, st)
                               : scanbwd::dispatch<__nv_bfloat16>(p, zm, f.delta_softplus != 0, st);
}
