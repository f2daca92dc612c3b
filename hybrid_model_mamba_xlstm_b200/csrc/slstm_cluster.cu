// slstm_cluster.cu — persistent sLSTM recurrence, one 8-CTA cluster per head.
//
// Each CTA of the cluster owns hd/8 channels (all four gates of them): its
// slice of the block-diagonal recurrent weights R[head] (hd x hd/2 bf16,
// 64 KB at hd = 256) is loaded ONCE into registers as mma.sync A fragments,
// so every step's R^T h_{t-1} for up to 8 batch rows is a handful of
// register-resident m16n8k16 MMAs.  The per-channel exponential-gate
// stabilizer m and the cell live in registers, one (channel, batch row) per
// thread.  The RMSNorm over head_dim couples the CTAs; each step makes two
// small cluster exchanges with st.async stores that complete transaction
// bytes on the receiver's mbarrier (no separate signal):
//   1. per batch row, this CTA's (max m, sum of squares of its stabilized
//      cells) — 8 bytes per row to every CTA;
//   2. after combining the 8 partials into the row's norm, h of this CTA's
//      channels as bf16, written straight into every CTA's MMA operand.
// Waits are bounded (error flag + early exit, no hang).
#include <cuda_bf16.h>

#include <cstdlib>

#include "capi_internal.h"
#include "common.cuh"
#include "slstm.h"

namespace hxm {
namespace slstm {

constexpr int kCL = 8;        // CTAs per cluster (one head)
constexpr int kBR = 8;        // batch rows per cluster (mma N)
constexpr int kRing = 2;      // gate pre-activation slots (current, next step)

// log(sigmoid(x)) = min(x, 0) - log1p(exp(-|x|)), the log1p on the MUFU pipe
// as ln2 * lg2(1 + 2^(-|x| log2 e)) (absolute error ~1e-7)
HXM_DEV float log_sigmoid_f(float x) {
  return fminf(x, 0.f) - kLn2 * lg2_approx(1.f + ex2_approx(-fabsf(x) * kLog2e));
}

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
// Stores into a peer CTA's shared memory that complete their byte count of
// transaction on the peer's mbarrier (no separate signal needed).
HXM_DEV void st_async_v2(uint32_t raddr, float2 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(raddr),
               "f"(v.x), "f"(v.y), "r"(rbar)
               : "memory");
}
HXM_DEV void st_async_v4u(uint32_t raddr, uint4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
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
// Bounded wait on phase `parity`: false if it gave up after `limit` SM cycles
// (the caller's wait_limit_cycles; 4e9 ~ 2 s by default).
HXM_DEV bool wait_bounded(uint64_t* bar, uint32_t parity, long long limit) {
  if (try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!try_wait_cluster(bar, parity))
    if (clock64() - t0 > limit) return false;
  return true;
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
  static_assert(kCPC * kBR == kNT, "one (channel, batch row) pair per thread");
  static_assert(kCPC >= 8 && kCPC <= 32, "a batch row's channels sit in one warp, in groups of 8");
  static constexpr int kHP = HD + 8;          // bf16 row pitch of the MMA operand (16-byte multiple)
  // shared memory (bytes)
  static constexpr int kH = 0;                                       // bf16 [kBR][kHP]
  static constexpr int kPart = kH + kBR * kHP * 2;                   // float2 [kCL][kBR]
  static constexpr int kPre = kPart + kCL * kBR * 8;                 // float [kBR][kCols]
  static constexpr int kG = kPre + kBR * kCols * 4;                  // float [kRing][kBR][4][kCPC]
  static constexpr int kW = kG + kRing * kBR * 4 * kCPC * 4;         // float [HD]
  static constexpr int kBar = kW + HD * 4;                           // 2 x uint64
  static constexpr int kBytes = kBar + 32;
  static constexpr uint32_t kPartTx = kCL * kBR * 8;                 // bytes per exchange-1 phase
  static constexpr uint32_t kHTx = kBR * HD * 2;                     // bytes per exchange-2 phase
  static_assert(kH % 16 == 0 && kPart % 16 == 0 && (kHP * 2) % 16 == 0, "st.async alignment");
};

// HPC heads per cluster: 1, or 2 for small batches (at most kBR / 2 rows), where the kBR
// (head, row) slots of the MMA's N dimension hold two heads' rows: every warp then runs both
// heads' R fragments (twice the registers and MMAs, each head's columns kept) and a layer
// occupies half the SMs — at batch 1 the 6 sLSTM layers of a prefill wavefront then fit on
// the GPU at once beside the other layers.
template <typename T, int HD, int HPC>
__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(HD, 1) slstm_cluster_kernel(const Params p) {
  using L = CL<HD>;
  constexpr int kRows = kBR / HPC;  // batch rows per head in one cluster
  static_assert(L::kMW == 1, "one m-tile per warp");
  extern __shared__ __align__(16) unsigned char sm[];
  __nv_bfloat16* hprev = reinterpret_cast<__nv_bfloat16*>(sm + L::kH);
  float2* part = reinterpret_cast<float2*>(sm + L::kPart);
  float* pre = reinterpret_cast<float*>(sm + L::kPre);
  float* gring = reinterpret_cast<float*>(sm + L::kG);
  float* wsm = reinterpret_cast<float*>(sm + L::kW);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBar);  // [0] partials, [1] h

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster_rank();
  const int head0 = blockIdx.x / kCL * HPC;
  const int b0 = blockIdx.y * kRows;
  const int nb = min(kRows, p.batch - b0);
  const int c0 = rank * L::kCPC;  // first channel of this CTA
  // this thread's (channel, slot) pair: a slot's kCPC channels are kCPC consecutive lanes;
  // slot bl = (head head0 + bl / kRows, batch row b0 + bl % kRows)
  const int c = tid % L::kCPC, bl = tid / L::kCPC;
  const int head = head0 + bl / kRows, brow = bl % kRows;
  const bool live = brow < nb;

  // ---- R slice -> mma A fragments (registers), once ------------------------------
  // local column m = q*kCPC + c  <->  R[head][k][q*HD + c0 + c]
  uint32_t afr[HPC][L::kKT][4];
  {
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int mw = 0; mw < HPC; ++mw) {
      const __nv_bfloat16* R = p.R + (int64_t)(head0 + mw) * HD * 4 * HD;
      const int mt = warp;
#pragma unroll
      for (int kt = 0; kt < L::kKT; ++kt) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int m = mt * 16 + g + ((r & 1) ? 8 : 0);
          const int k = kt * 16 + t4 * 2 + ((r & 2) ? 8 : 0);
          const int q = m / L::kCPC, cc = m % L::kCPC;
          const int64_t col = (int64_t)q * HD + c0 + cc;
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
    const int r = e / HD, j = e % HD;
    float hv = 0.f;
    if (r % kRows < nb && p.h0) hv = p.h0[((int64_t)(b0 + r % kRows) * p.heads + head0 + r / kRows) * HD + j];
    hprev[r * L::kHP + j] = __float2bfloat16_rn(hv);
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&bars[0])), "r"(1) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&bars[1])), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // each phase = one local arrive (with the byte expectation) + the peers'
    // st.async bytes; phase 0 of both is armed before the start-up cluster
    // barrier, so no peer data can precede its arm.
    arm_tx(&bars[0], L::kPartTx);
    arm_tx(&bars[1], L::kHTx);
  }
  // stabilized cell and its log-scale for this thread's pair
  float cs = (live && p.c0) ? p.c0[((int64_t)(b0 + brow) * p.heads + head) * HD + c0 + c] : 0.f;
  float ms = 0.f;
  const float wc = p.w[c0 + c];
  const T* gsrc = static_cast<const T*>(p.gates);
  // gate pre-activations of step t: element e = (row, q, channel) of this CTA's slice
  constexpr int kGE = (kBR * 4 * L::kCPC) / L::kNT;
  auto fetch_gates = [&](int t, float (&v)[kGE]) {
#pragma unroll
    for (int i = 0; i < kGE; ++i) {
      const int e = tid + i * L::kNT;
      const int cc = e % L::kCPC, q = (e / L::kCPC) % 4, r = e / (4 * L::kCPC);
      const int rr = r % kRows, hh = head0 + r / kRows;
      v[i] = (rr < nb && t < p.seqlen)
                 ? to_f32<T>(gsrc[(((int64_t)(b0 + rr) * p.seqlen + t) * p.heads + hh) * 4 * HD + q * HD + c0 + cc])
                 : 0.f;
    }
  };
  auto store_gates = [&](int t, const float (&v)[kGE]) {
    float* dst = gring + (t % kRing) * kBR * 4 * L::kCPC;
#pragma unroll
    for (int i = 0; i < kGE; ++i) dst[tid + i * L::kNT] = v[i];
  };
  {
    float v[kGE];
    fetch_gates(0, v);
    store_gates(0, v);
  }
  __syncthreads();
  cluster_sync();  // every CTA's barriers initialized before any remote arrive

  const uint32_t part_addr = smem_u32(part + rank * kBR + bl);                 // my slot in every peer
  const uint32_t h_addr = smem_u32(hprev + bl * L::kHP + c0 + c);              // my channels in every peer
  const uint32_t bar_part = smem_u32(&bars[0]), bar_h = smem_u32(&bars[1]);
  T* hout = static_cast<T*>(p.h_out);
  bool bad = false;
  float hlast = 0.f;
  // wait_limit < 0 (the error-path test): wait -wait_limit cycles on step 0's partials before
  // any CTA has sent them, so the wait runs out with no exchange in flight
  if (p.wait_limit < 0) bad = !wait_bounded(&bars[0], 0, -p.wait_limit);
  if (__syncthreads_or(bad)) bad = true;

  for (int t = 0; !bad && t < p.seqlen; ++t) {
    const uint32_t parity = t & 1;
    float gnext[kGE];
    fetch_gates(t + 1, gnext);  // consumed at the end of the step: latency hidden behind the step
    // (a) gate pre-activations R^T h_{t-1}: D[m][n] (m = gate column, n = batch row), 4 MMA chains
    {
      const int g = lane >> 2, t4 = lane & 3;
      // D[m][n] (n = slot): with two heads, each head's MMA covers all 8 slots and this
      // thread keeps the head of its own slots 2 t4, 2 t4 + 1 (both of head t4 / 2)
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int mw = 0; mw < HPC; ++mw) {
        float acc[4][4] = {};
#pragma unroll
        for (int kt = 0; kt < L::kKT; ++kt) {
          const __nv_bfloat16* hb = hprev + g * L::kHP + kt * 16 + t4 * 2;
          const uint32_t b0r = *reinterpret_cast<const uint32_t*>(hb);
          const uint32_t b1r = *reinterpret_cast<const uint32_t*>(hb + 8);
          mma_16816(acc[kt & 3], afr[mw][kt], b0r, b1r);
        }
        if (HPC == 1 || mw == (2 * t4) / kRows) {
#pragma unroll
          for (int r = 0; r < 4; ++r) d[r] = (acc[0][r] + acc[1][r]) + (acc[2][r] + acc[3][r]);
        }
      }
      {
        const int m = warp * 16 + g;
        pre[(2 * t4) * L::kCols + m] = d[0];
        pre[(2 * t4 + 1) * L::kCols + m] = d[1];
        pre[(2 * t4) * L::kCols + m + 8] = d[2];
        pre[(2 * t4 + 1) * L::kCols + m + 8] = d[3];
      }
    }
    __syncthreads();
    // (b) cell update of this thread's pair; per-row partial (max m, sum of squares) to every CTA
    float og;
    {
      const float* gt = gring + (t % kRing) * kBR * 4 * L::kCPC;
      float gp[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) gp[q] = pre[bl * L::kCols + q * L::kCPC + c] + gt[(bl * 4 + q) * L::kCPC + c];
      const float lf = log_sigmoid_f(gp[1]);
      const float li = p.exp_gate ? gp[0] : log_sigmoid_f(gp[0]);
      const float mn = fmaxf(ms + lf, li);
      cs = ex2_approx((ms + lf - mn) * kLog2e) * cs + ex2_approx((li - mn) * kLog2e) * tanh_approx(gp[3]);
      ms = mn;
      og = fmaf(0.5f, tanh_approx(0.5f * gp[2]), 0.5f);
      float mloc = ms;
#pragma unroll
      for (int o = L::kCPC / 2; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
      const float sc = ex2_approx((ms - mloc) * kLog2e) * cs;
      float sloc = sc * sc;
#pragma unroll
      for (int o = L::kCPC / 2; o > 0; o >>= 1) sloc += __shfl_xor_sync(0xffffffffu, sloc, o);
      if (c == 0) {
#pragma unroll
        for (int r = 0; r < kCL; ++r)
          st_async_v2(map_to_rank(part_addr, r), make_float2(mloc, sloc), map_to_rank(bar_part, r));
      }
    }
    // (c) wait for the 8 partials of every row (bounded), then re-arm for step
    //     t + 1 before the barrier below: peers send step t + 1 partials only
    //     after their step t + 1 MMA, which needs this CTA's step t h, sent
    //     after that barrier.
    bad = !wait_bounded(&bars[0], parity, p.wait_limit);
    if (tid == 0 && !bad && t + 1 < p.seqlen) arm_tx(&bars[0], L::kPartTx);
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    // (d) the row's norm from the 8 partials; h of this pair; bf16 h of 8
    //     consecutive channels to every CTA's MMA operand
    {
      float M = -INFINITY;
#pragma unroll
      for (int k = 0; k < kCL; ++k) M = fmaxf(M, part[k * kBR + bl].x);
      float S = 0.f;
#pragma unroll
      for (int k = 0; k < kCL; ++k) {
        const float2 pk = part[k * kBR + bl];
        const float e = ex2_approx((pk.x - M) * kLog2e);
        S = fmaf(e * e, pk.y, S);
      }
      const float rinv = rsqrtf(S / HD + p.eps * ex2_approx(-2.f * M * kLog2e));
      const float hv = og * tanh_approx(wc * ex2_approx((ms - M) * kLog2e) * cs * rinv);
      hlast = hv;
      if (live) hout[(((int64_t)(b0 + brow) * p.seqlen + t) * p.heads + head) * HD + c0 + c] = from_f32<T>(hv);
      // pack: lane pairs -> bf16x2, then 4 pairs -> 16 bytes at the group's first lane
      const float hn = __shfl_down_sync(0xffffffffu, hv, 1);
      __nv_bfloat162 pr = __floats2bfloat162_rn(hv, hn);
      const uint32_t w0 = *reinterpret_cast<uint32_t*>(&pr);
      const uint32_t w1 = __shfl_down_sync(0xffffffffu, w0, 2);
      const uint32_t w2 = __shfl_down_sync(0xffffffffu, w0, 4);
      const uint32_t w3 = __shfl_down_sync(0xffffffffu, w0, 6);
      if ((c & 7) == 0) {
        const uint4 v = make_uint4(w0, w1, w2, w3);
#pragma unroll
        for (int r = 0; r < kCL; ++r) st_async_v4u(map_to_rank(h_addr, r), v, map_to_rank(bar_h, r));
      }
    }
    store_gates(t + 1, gnext);
    // (e) wait for every CTA's h (bounded); it lands directly in hprev.  Re-arm
    //     for step t + 1 first: peers send step t + 1 h only after this CTA's
    //     step t + 1 partials, sent after the barrier below.
    bad = !wait_bounded(&bars[1], parity, p.wait_limit);
    if (tid == 0 && !bad && t + 1 < p.seqlen) arm_tx(&bars[1], L::kHTx);
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
  }

  if (!bad) {
    if (p.hT && live) p.hT[((int64_t)(b0 + brow) * p.heads + head) * HD + c0 + c] = hlast;
    if (p.cT && live) p.cT[((int64_t)(b0 + brow) * p.heads + head) * HD + c0 + c] = ex2_approx(ms * kLog2e) * cs;
  } else if (tid == 0 && p.error_flag) {
    atomicExch(p.error_flag, 1);
  }
  cluster_sync();  // no CTA leaves while peers may still write into its shared memory
}

template <typename T, int HD, int HPC>
static hxm_status launch_hpc(const Params& p, cudaStream_t st) {
  using L = CL<HD>;
  auto kern = slstm_cluster_kernel<T, HD, HPC>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
  constexpr int kRows = kBR / HPC;
  dim3 grid(kCL * p.heads / HPC, (p.batch + kRows - 1) / kRows);
  kern<<<grid, L::kNT, L::kBytes, st>>>(p);
  return check_launch("hxm_slstm_scan_fwd (cluster)");
}
// Two heads per cluster when every cluster then still holds all its rows (batch <= kBR / 2) and
// the heads pair up; HXM_SLSTM_HPC = 1 | 2 overrides (2 only where it applies).
template <typename T, int HD>
static hxm_status launch_hd(const Params& p, cudaStream_t st) {
  const char* knob = std::getenv("HXM_SLSTM_HPC");
  int hpc = knob ? std::atoi(knob) : 0;
  const bool pairable = p.heads % 2 == 0 && p.batch <= kBR / 2;
  if (hpc != 1 && hpc != 2) hpc = pairable ? 2 : 1;
  if (hpc == 2 && pairable) return launch_hpc<T, HD, 2>(p, st);
  return launch_hpc<T, HD, 1>(p, st);
}

hxm_status launch_cluster(const Params& p, cudaStream_t st) {
  if (!p.R || (p.hd != 128 && p.hd != 256)) return HXM_EUNSUPPORTED;
  if (p.io_dtype == HXM_F32) return p.hd == 128 ? launch_hd<float, 128>(p, st) : launch_hd<float, 256>(p, st);
  return p.hd == 128 ? launch_hd<__nv_bfloat16, 128>(p, st) : launch_hd<__nv_bfloat16, 256>(p, st);
}

}  // namespace slstm
}  // namespace hxm
