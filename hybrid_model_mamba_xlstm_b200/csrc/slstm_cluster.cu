// slstm_cluster.cu — persistent sLSTM recurrence, one 8-CTA cluster per head.
//
// Each CTA of the cluster owns hd/8 channels (all four gates of them): its
// slice of the block-diagonal recurrent weights R[head] (hd x hd/2 bf16,
// 64 KB at hd = 256) is loaded ONCE into registers as mma.sync A fragments,
// so every step's R^T h_{t-1} for up to 8 batch rows is a handful of
// register-resident m16n8k16 MMAs.  The per-channel exponential-gate
// stabilizer m and the cell live in registers.  After the cell update each
// CTA broadcasts (cell, m, o) of its channels into every CTA's shared memory
// with st.async stores that complete transaction bytes on the receiver's
// mbarrier (no separate signal); every CTA then has all hd channels and finishes the
// RMSNorm over head_dim and h = o*tanh(.) locally — one cluster exchange per
// step.  Waits are bounded (error flag + early exit, no hang).
#include <cuda_bf16.h>

#include "capi_internal.h"
#include "common.cuh"
#include "slstm.h"

namespace hxm {
namespace slstm {

constexpr int kCL = 8;        // CTAs per cluster (one head)
constexpr int kBR = 8;        // batch rows per cluster (mma N)
constexpr int kRing = 2;      // gate pre-activation slots (current, next step)

HXM_DEV float log_sigmoid_f(float x) { return fminf(x, 0.f) - log1pf(__expf(-fabsf(x))); }

HXM_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HXM_DEV uint32_t map_to_rank(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}
// 16-byte store into a peer CTA's shared memory that completes 16 bytes of
// transaction count on the peer's mbarrier (no separate signal needed).
HXM_DEV void st_async_v4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
               : "memory");
}
HXM_DEV void arm_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
HXM_DEV bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
HXM_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
HXM_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
struct CL {
  static constexpr int kCPC = HD / kCL;       // channels per CTA
  static constexpr int kCols = 4 * kCPC;      // gate columns per CTA
  static constexpr int kMT = kCols / 16;      // m-tiles
  static constexpr int kKT = HD / 16;         // k-tiles
  static constexpr int kNT = HD;              // threads per CTA (one m-tile per warp)
  static constexpr int kMW = kMT / (kNT / 32);  // m-tiles per warp (= 1)
  static constexpr int kTPB = kNT / kBR;      // threads per batch row in the norm phase
  static constexpr int kCPT = HD / kTPB;      // channels per thread in the norm phase
  static constexpr int kPairs = kCPC * kBR;   // (channel, batch) pairs per CTA
  static constexpr int kPPT = kPairs / kNT;
  // shared memory (bytes)
  static constexpr int kX = 0;                                       // float4 [2][kBR][HD]
  static constexpr int kH = kX + 2 * kBR * HD * 16;                  // bf16 [kBR][HD + 8]
  static constexpr int kPre = kH + kBR * (HD + 8) * 2;               // float [kBR][kCols]
  static constexpr int kG = kPre + kBR * kCols * 4;                  // float [kRing][kBR][4][kCPC]
  static constexpr int kW = kG + kRing * kBR * 4 * kCPC * 4;         // float [HD]
  static constexpr int kBar = kW + HD * 4;                           // 2 x uint64
  static constexpr int kBytes = kBar + 32;
};

template <typename T, int HD>
__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(HD, 1) slstm_cluster_kernel(const Params p) {
  using L = CL<HD>;
  extern __shared__ __align__(16) unsigned char sm[];
  float4* xbuf = reinterpret_cast<float4*>(sm + L::kX);
  __nv_bfloat16* hprev = reinterpret_cast<__nv_bfloat16*>(sm + L::kH);
  float* pre = reinterpret_cast<float*>(sm + L::kPre);
  float* gring = reinterpret_cast<float*>(sm + L::kG);
  float* wsm = reinterpret_cast<float*>(sm + L::kW);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBar);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster_rank();
  const int head = blockIdx.x / kCL;
  const int b0 = blockIdx.y * kBR;
  const int nb = min(kBR, p.batch - b0);
  const int HDs = HD;
  const int c0 = rank * L::kCPC;  // first channel of this CTA

  // ---- R slice -> mma A fragments (registers), once ------------------------------
  // local column m = q*kCPC + c  <->  R[head][k][q*HD + c0 + c]
  uint32_t afr[L::kMW][L::kKT][4];
  {
    const __nv_bfloat16* R = p.R + (int64_t)head * HD * 4 * HD;
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int mw = 0; mw < L::kMW; ++mw) {
      const int mt = warp * L::kMW + mw;
#pragma unroll
      for (int kt = 0; kt < L::kKT; ++kt) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int m = mt * 16 + g + ((r & 1) ? 8 : 0);
          const int k = kt * 16 + t4 * 2 + ((r & 2) ? 8 : 0);
          const int q = m / L::kCPC, c = m % L::kCPC;
          const int64_t col = (int64_t)q * HD + c0 + c;
          __nv_bfloat162 v;
          v.x = R[(int64_t)k * 4 * HD + col];
          v.y = R[(int64_t)(k + 1) * 4 * HD + col];
          afr[mw][kt][r] = *reinterpret_cast<uint32_t*>(&v);
        }
      }
    }
  }
  for (int j = tid; j < HD; j += L::kNT) wsm[j] = p.w[j];
  // initial h (bf16 operand) for all channels
  for (int e = tid; e < kBR * HD; e += L::kNT) {
    const int bl = e / HD, j = e % HD;
    float hv = 0.f;
    if (bl < nb && p.h0) hv = p.h0[((int64_t)(b0 + bl) * p.heads + head) * HD + j];
    hprev[bl * (HD + 8) + j] = __float2bfloat16_rn(hv);
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&bars[0])), "r"(1) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&bars[1])), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // each phase = one local arrive (with the byte expectation) + kBR*HD*16
    // bytes of st.async stores from the 8 CTAs; arm steps 0 and 1 before the
    // start-up cluster barrier so no peer data can precede its arm.
    arm_tx(&bars[0], kBR * HD * 16);
    arm_tx(&bars[1], kBR * HD * 16);
  }
  // per-thread (channel, batch) pairs: stabilized cell and its log-scale
  float cs[L::kPPT], ms[L::kPPT];
#pragma unroll
  for (int i = 0; i < L::kPPT; ++i) {
    const int pi = tid + i * L::kNT;
    const int c = pi % L::kCPC, bl = pi / L::kCPC;
    cs[i] = (bl < nb && p.c0) ? p.c0[((int64_t)(b0 + bl) * p.heads + head) * HD + c0 + c] : 0.f;
    ms[i] = 0.f;
  }
  const T* gsrc = static_cast<const T*>(p.gates);
  // gate pre-activations of step t: element e = (bl, q, c) of this CTA's slice
  constexpr int kGE = (kBR * 4 * L::kCPC) / L::kNT;
  auto fetch_gates = [&](int t, float (&v)[kGE]) {
#pragma unroll
    for (int i = 0; i < kGE; ++i) {
      const int e = tid + i * L::kNT;
      const int c = e % L::kCPC, q = (e / L::kCPC) % 4, bl = e / (4 * L::kCPC);
      v[i] = (bl < nb && t < p.seqlen)
                 ? to_f32<T>(gsrc[(((int64_t)(b0 + bl) * p.seqlen + t) * p.heads + head) * 4 * HD + q * HD + c0 + c])
                 : 0.f;
    }
  };
  auto store_gates = [&](int t, const float (&v)[kGE]) {
    float* dst = gring + (t % kRing) * kBR * 4 * L::kCPC;
#pragma unroll
    for (int i = 0; i < kGE; ++i) dst[tid + i * L::kNT] = v[i];
  };
  auto load_gates = [&](int t) {
    float v[kGE];
    fetch_gates(t, v);
    store_gates(t, v);
  };
  load_gates(0);
  __syncthreads();
  cluster_sync();  // every CTA's barriers initialized before any remote arrive

  uint32_t xaddr0 = smem_u32(xbuf);
  uint32_t baddr0 = smem_u32(&bars[0]);
  T* hout = static_cast<T*>(p.h_out);
  bool bad = false;
  float hlast[L::kCPT];
#pragma unroll
  for (int i = 0; i < L::kCPT; ++i) hlast[i] = 0.f;

  for (int t = 0; t < p.seqlen; ++t) {
    const int par = t & 1;
    float gnext[kGE];
    fetch_gates(t + 1, gnext);  // consumed at the end of the step: latency hidden behind the step
    // (a) gate pre-activations R^T h_{t-1}: D[m][n] (m = gate column, n = batch row)
    {
      const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
      for (int mw = 0; mw < L::kMW; ++mw) {
        float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // two independent chains
#pragma unroll
        for (int kt = 0; kt < L::kKT; ++kt) {
          const __nv_bfloat16* hb = hprev + g * (HD + 8) + kt * 16 + t4 * 2;
          const uint32_t b0r = *reinterpret_cast<const uint32_t*>(hb);
          const uint32_t b1r = *reinterpret_cast<const uint32_t*>(hb + 8);
          if (kt & 1) mma_16816(e, afr[mw][kt], b0r, b1r);
          else mma_16816(d, afr[mw][kt], b0r, b1r);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) d[r] += e[r];
        const int m = (warp * L::kMW + mw) * 16 + g;
        pre[(2 * t4) * L::kCols + m] = d[0];
        pre[(2 * t4 + 1) * L::kCols + m] = d[1];
        pre[(2 * t4) * L::kCols + m + 8] = d[2];
        pre[(2 * t4 + 1) * L::kCols + m + 8] = d[3];
      }
    }
    __syncthreads();
    // (b) cell update of own (channel, batch) pairs; broadcast (cell, m, o) to the cluster
    {
      const float* gt = gring + (t % kRing) * kBR * 4 * L::kCPC;
#pragma unroll
      for (int i = 0; i < L::kPPT; ++i) {
        const int pi = tid + i * L::kNT;
        const int c = pi % L::kCPC, bl = pi / L::kCPC;
        float gp[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) gp[q] = pre[bl * L::kCols + q * L::kCPC + c] + gt[(bl * 4 + q) * L::kCPC + c];
        const float lf = log_sigmoid_f(gp[1]);
        const float li = p.exp_gate ? gp[0] : log_sigmoid_f(gp[0]);
        const float mn = fmaxf(ms[i] + lf, li);
        cs[i] = __expf(ms[i] + lf - mn) * cs[i] + __expf(li - mn) * tanh_approx(gp[3]);
        ms[i] = mn;
        const float og = fmaf(0.5f, tanh_approx(0.5f * gp[2]), 0.5f);
        const float4 v = make_float4(cs[i], ms[i], og, 0.f);
        const uint32_t off = (uint32_t)(((par * kBR + bl) * HDs + c0 + c) * 16);
#pragma unroll
        for (int r = 0; r < kCL; ++r) st_async_v4(map_to_rank(xaddr0 + off, r), v, map_to_rank(baddr0 + par * 8, r));
      }
    }
    // (c) wait for all 8 slices (bounded)
    {
      const uint32_t parity = (t >> 1) & 1;
      if (!try_wait_cluster(&bars[par], parity)) {
        const long long t0 = clock64();
        while (!try_wait_cluster(&bars[par], parity)) {
          if (clock64() - t0 > 4000000000ll) {
            bad = true;
            break;
          }
        }
      }
    }
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    // re-arm this buffer's barrier for step t + 2.  Peers can only send step
    // t + 2 after waiting on step t + 1, which needs this CTA's step t + 1
    // stores — issued after this point — so the arm always precedes the data.
    if (tid == 0 && t + 2 < p.seqlen) arm_tx(&bars[par], kBR * HD * 16);
    // (d) RMSNorm over head_dim and h for every channel (kTPB threads per batch row)
    {
      const int bl = tid / L::kTPB, sub = tid % L::kTPB;
      const float4* xr = xbuf + (par * kBR + bl) * HD;
      float M = -INFINITY;
#pragma unroll
      for (int i = 0; i < L::kCPT; ++i) M = fmaxf(M, xr[sub + L::kTPB * i].y);
#pragma unroll
      for (int o = L::kTPB / 2; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      float S = 0.f;
#pragma unroll
      for (int i = 0; i < L::kCPT; ++i) {
        const float4 x = xr[sub + L::kTPB * i];
        const float sc = __expf(x.y - M) * x.x;
        S = fmaf(sc, sc, S);
      }
#pragma unroll
      for (int o = L::kTPB / 2; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
      const float rinv = rsqrtf(S / HD + p.eps * __expf(-2.f * M));
#pragma unroll
      for (int i = 0; i < L::kCPT; ++i) {
        const int j = sub + L::kTPB * i;
        const float4 x = xr[j];
        const float hv = x.z * tanh_approx(wsm[j] * __expf(x.y - M) * x.x * rinv);
        hprev[bl * (HD + 8) + j] = __float2bfloat16_rn(hv);
        hlast[i] = hv;
        if (bl < nb && j >= c0 && j < c0 + L::kCPC)
          hout[(((int64_t)(b0 + bl) * p.seqlen + t) * p.heads + head) * HD + j] = from_f32<T>(hv);
      }
    }
    store_gates(t + 1, gnext);
    __syncthreads();
  }

  if (!bad) {
    const int bl = tid / L::kTPB, sub = tid % L::kTPB;
    if (p.hT && bl < nb) {
#pragma unroll
      for (int i = 0; i < L::kCPT; ++i) {
        const int j = sub + L::kTPB * i;
        if (j >= c0 && j < c0 + L::kCPC) p.hT[((int64_t)(b0 + bl) * p.heads + head) * HD + j] = hlast[i];
      }
    }
    if (p.cT) {
#pragma unroll
      for (int i = 0; i < L::kPPT; ++i) {
        const int pi = tid + i * L::kNT;
        const int c = pi % L::kCPC, bl2 = pi / L::kCPC;
        if (bl2 < nb) p.cT[((int64_t)(b0 + bl2) * p.heads + head) * HD + c0 + c] = __expf(ms[i]) * cs[i];
      }
    }
  } else if (tid == 0 && p.error_flag) {
    atomicExch(p.error_flag, 1);
  }
  cluster_sync();  // no CTA leaves while peers may still write into its shared memory
}

template <typename T, int HD>
static hxm_status launch_hd(const Params& p, cudaStream_t st) {
  using L = CL<HD>;
  auto kern = slstm_cluster_kernel<T, HD>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  dim3 grid(kCL * p.heads, (p.batch + kBR - 1) / kBR);
  kern<<<grid, L::kNT, L::kBytes, st>>>(p);
  return check_launch("hxm_slstm_scan_fwd (cluster)");
}

hxm_status launch_cluster(const Params& p, cudaStream_t st) {
  if (!p.R || (p.hd != 128 && p.hd != 256)) return HXM_EUNSUPPORTED;
  if (p.io_dtype == HXM_F32) return p.hd == 128 ? launch_hd<float, 128>(p, st) : launch_hd<float, 256>(p, st);
  return p.hd == 128 ? launch_hd<__nv_bfloat16, 128>(p, st) : launch_hd<__nv_bfloat16, 256>(p, st);
}

}  // namespace slstm
}  // namespace hxm
