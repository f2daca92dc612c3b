// mlstm_stream.cu — chunkwise mLSTM on tcgen05 for per-channel gates and for
// dqk up to 512, streaming the key dimension through shared memory.
//
// Two kernels:
//  1. mlstm_prescale_kernel (CUDA cores, one pass over q, k, gates): per chunk
//     of 128 steps and key channel j, with b_t[j] = sum_{s<=t} log f_s[j] inside
//     the chunk, g[j] = b_127[j] and the midpoint rho[j] = g[j] / 2:
//        Qs[t,j] = q[t,j] e^(b_t - rho)              (|exponent| <= |g|/2)
//        Ks[s,j] = k[s,j] e^(rho - b_s + log i_s)
//        Kh[s,j] = k[s,j] e^(g - b_s + log i_s)
//        decay[j] = e^g,  rho_e[j] = e^rho
//     so that  sum_j q_t k_s e^(b_t - b_s + log i_s) = Qs_t . Ks_s  (intra-chunk)
//     and      state' = diag(e^g) state + Kh^T v       (inter-chunk), the
//     recurrence of tfla_forward_pytorch (tfla_interface.py:113-137) with
//     gates multiplying along the key dimension (mlstm_block.py:117-129).
//  2. mlstm_stream_kernel (tcgen05): per (b, h, 64-wide value tile), per chunk
//        S  = Qs Ks^T, H = Qs (rho_e . state) + causal(S) V     (TMEM)
//        qn = Qs (rho_e . n) on CUDA cores,  den = qn + rowsum(causal S)
//        h  = H / max(den, 1)
//        state = decay . state + Kh^T V,  n = decay . n + Kh^T 1   (TMEM)
//     Q/K panels (64 key channels) stream through a 3-stage TMA ring; the state
//     (dqk x 64 fp32) and n live in TMEM.  No overflow as long as the total
//     log forget gate of one 128-step chunk stays above about -160 per channel
//     (exponents are bounded by half of it); the reference itself overflows
//     for input-gate pre-activations above ~88 and so does this kernel.
#include "capi_internal.h"
#include "common.cuh"
#include "mlstm.h"
#include "tc_sm100.cuh"
#include "tma_host.h"

namespace hxm {
namespace mlstm {

constexpr int kC = 128;
constexpr int kDV = 64;
constexpr int kPanel = 16384;
constexpr int kStages = 3;

// ---------------------------------------------------------------- pre-pass --
// grid (B*H*nchunks, ceil(DK/128)), block 128: thread = key channel j.
template <typename T>
__global__ void __launch_bounds__(128) mlstm_prescale_kernel(const Params p, __nv_bfloat16* Qs, __nv_bfloat16* Ks,
                                                             __nv_bfloat16* Kh, float* decay, float* rho_e) {
  const int nch = (p.seqlen + kC - 1) / kC;
  const int c = blockIdx.x % nch;
  const int bh = blockIdx.x / nch;
  const int b = bh / p.heads, h = bh % p.heads;
  const int j = blockIdx.y * 128 + threadIdx.x;
  if (j >= p.dqk) return;
  const int t0 = c * kC, tn = min(kC, p.seqlen - t0);
  const T* q = static_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
  const T* k = static_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
  const float* li = p.log_i + b * p.si[0] + h * p.si[1];
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1];
  const bool pc = p.gate_mode == 1;
  const int gj = pc ? j : 0;
  float g = 0.f;
  for (int t = 0; t < tn; ++t) g += lf[(int64_t)(t0 + t) * p.tf + gj];
  const float rho = 0.5f * g;
  const int64_t ob = (int64_t)bh * p.seqlen * p.dqk;
  float bt = 0.f;
  for (int t = 0; t < tn; ++t) {
    const int64_t tt = t0 + t;
    bt += lf[tt * p.tf + gj];
    const float lit = li[tt * p.ti + gj];
    const float qv = to_f32<T>(q[tt * p.tq + j]);
    const float kv = to_f32<T>(k[tt * p.tk + j]);
    Qs[ob + tt * p.dqk + j] = __float2bfloat16_rn(qv * __expf(bt - rho));
    Ks[ob + tt * p.dqk + j] = __float2bfloat16_rn(kv * __expf(rho - bt + lit));
    Kh[ob + tt * p.dqk + j] = __float2bfloat16_rn(kv * __expf(g - bt + lit));
  }
  decay[((int64_t)bh * nch + c) * p.dqk + j] = __expf(g);
  rho_e[((int64_t)bh * nch + c) * p.dqk + j] = __expf(rho);
}

// ------------------------------------------------------------ stream kernel --
template <int DK>
struct SL {
  static constexpr int kNP = DK / 64;                 // key panels
  static constexpr int kNB = DK / 128;                // state row blocks (TMEM 128 lanes)
  static constexpr int kRing = 0;                     // kStages x 32 KB
  static constexpr int kSnap = kRing + kStages * 2 * kPanel;  // DK rows x 128 B (MN-major B, one 64-wide N panel)
  static constexpr int kP = kSnap + DK * 128;         // 2 panels
  static constexpr int kV = kP + 2 * kPanel;          // 1 panel
  static constexpr int kOnes = kV + kPanel;           // K-major [16][128] = 2 x 2 KB
  static constexpr int kNs = kOnes + 4096;            // float [DK]  rho_e . n   (for qn)
  static constexpr int kBar = kNs + DK * 4;           // full[kStages], empty[kStages], v, s, h, acc
  static constexpr int kSlot = kBar + 8 * (2 * kStages + 4);
  static constexpr int kAbort = kSlot + 4;
  static constexpr int kBytes = kAbort + 12;
  // TMEM columns: S 0..127, H 128..191, state blocks 256 + 64 b, n blocks 192 + 16 b
  static constexpr int tS = 0, tH = 128, tN = 192, tAcc = 256;
  static_assert(tN + 16 * kNB <= tAcc && tAcc + 64 * kNB <= 512, "TMEM layout");
};

template <int DK>
__global__ void __launch_bounds__(128, 1)
    mlstm_stream_kernel(const __grid_constant__ CUtensorMap tmQs, const __grid_constant__ CUtensorMap tmKs,
                        const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmV,
                        const Params p, const float* __restrict__ decay, const float* __restrict__ rho_e) {
  using L = SL<DK>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint64_t* empty = full + kStages;
  uint64_t* bar_v = empty + kStages;
  uint64_t* bar_s = bar_v + 1;   // S and Qs.Snap done
  uint64_t* bar_h = bar_v + 2;   // P.V done
  uint64_t* bar_a = bar_v + 3;   // state update done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::kSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kAbort);
  float* ns = reinterpret_cast<float*>(sm + L::kNs);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e0 = blockIdx.x * kDV, h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.heads + h;
  const int nch = (p.seqlen + kC - 1) / kC;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1 + 4);  // MMA commit + one arrive per consumer warp
    }
    tc::mbar_init(bar_v, 1);
    tc::mbar_init(bar_s, 1);
    tc::mbar_init(bar_h, 1);
    tc::mbar_init(bar_a, 1);
    tc::fence_mbar_init();
    *abort_flag = 0;
  }
  {  // ones operand: K-major [16][128], row 0 = 1
    uint4* z = reinterpret_cast<uint4*>(sm + L::kOnes);
    for (int i = tid; i < 4096 / 16; i += 128) z[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    __nv_bfloat16* ones = reinterpret_cast<__nv_bfloat16*>(sm + L::kOnes);
    ones[((tid / 64) * 2048 + tc::sw128_offset(0, tid % 64)) / 2] = __float2bfloat16_rn(1.f);
  }
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *tmem_slot;

  // initial state -> TMEM (the caller's stabilized C0/n0 scaled by e^m0)
  const float s0 = p.m0 ? __expf(p.m0[bh]) : 1.f;
#pragma unroll 1
  for (int blk = 0; blk < L::kNB; ++blk) {
    const int row = blk * 128 + warp * 32 + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < kDV; c0 += 32) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = e0 + c0 + j;
        v[j] = (p.C0 && col < p.dv) ? s0 * p.C0[((int64_t)bh * DK + row) * p.dv + col] : 0.f;
      }
      tc::tmem_st32(tc::taddr(tm, warp * 32, L::tAcc + blk * 64 + c0), v);
    }
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    if (p.n0) v[0] = s0 * p.n0[(int64_t)bh * DK + row];
    tc::tmem_st16(tc::taddr(tm, warp * 32, L::tN + blk * 16), v);
  }
  tc::tmem_wait_st();

  // state (TMEM) -> rho_e(c)-scaled bf16 snapshot (smem) and rho_e . n (smem fp32)
  auto snapshot = [&](int c) {
    const float* re = rho_e + ((int64_t)bh * nch + c) * DK;
#pragma unroll 1
    for (int blk = 0; blk < L::kNB; ++blk) {
      const int row = blk * 128 + warp * 32 + lane;
      const float r = re[row];
#pragma unroll 1
      for (int c0 = 0; c0 < kDV; c0 += 32) {
        float v[32];
        tc::tmem_ld32(tc::taddr(tm, warp * 32, L::tAcc + blk * 64 + c0), v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack2<__nv_bfloat16>(r * v[8 * q + 0], r * v[8 * q + 1]);
          w.y = pack2<__nv_bfloat16>(r * v[8 * q + 2], r * v[8 * q + 3]);
          w.z = pack2<__nv_bfloat16>(r * v[8 * q + 4], r * v[8 * q + 5]);
          w.w = pack2<__nv_bfloat16>(r * v[8 * q + 6], r * v[8 * q + 7]);
          *reinterpret_cast<uint4*>(sm + L::kSnap + tc::sw128_offset(row, c0 + 8 * q)) = w;
        }
      }
      float v[16];
      tc::tmem_ld16(tc::taddr(tm, warp * 32, L::tN + blk * 16), v);
      tc::tmem_wait_ld();
      ns[row] = r * v[0];
    }
  };

  // producer state (thread 0): a global sequence of 32 KB stage loads
  //   per chunk: kNP panel loads (Qs_p + Ks_p) then kNB pair loads (Kh rows 128 blk ..)
  constexpr int kLoadsPerChunk = L::kNP + L::kNB;
  const int total_loads = nch * kLoadsPerChunk;
  int next_load = 0;
  auto issue_stage = [&](int idx) {
    const int slot = idx % kStages;
    const int c = idx / kLoadsPerChunk, r = idx % kLoadsPerChunk;
    unsigned char* dst = sm + L::kRing + slot * 2 * kPanel;
    tc::mbar_expect_tx(&full[slot], 2 * kPanel);
    const int t0 = c * kC;
    if (r < L::kNP) {
      tc::tma_load_4d(dst, &tmQs, &full[slot], r * 64, t0, h, b);
      tc::tma_load_4d(dst + kPanel, &tmKs, &full[slot], r * 64, t0, h, b);
    } else {
      const int blk = r - L::kNP;
      tc::tma_load_4d(dst, &tmKh, &full[slot], blk * 128, t0, h, b);
      tc::tma_load_4d(dst + kPanel, &tmKh, &full[slot], blk * 128 + 64, t0, h, b);
    }
  };
  // stage reuse: load idx >= kStages needs the consumers of load idx - kStages done
  auto produce_until = [&](int upto, bool& ok) {
    while (next_load < total_loads && next_load < upto) {
      if (next_load >= kStages) {
        const int prev = next_load - kStages;
        if (!tc::mbar_wait(&empty[prev % kStages], (prev / kStages) & 1, abort_flag)) { ok = false; return; }
      }
      issue_stage(next_load);
      ++next_load;
    }
  };

  snapshot(0);
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();

  constexpr uint32_t idS = tc::idesc_bf16(128, 128, false, false);
  constexpr uint32_t idH = tc::idesc_bf16(128, kDV, false, true);
  constexpr uint32_t idAcc = tc::idesc_bf16(128, kDV, true, true);
  constexpr uint32_t idN = tc::idesc_bf16(128, 16, true, false);

  bool okp = true;
  if (tid == 0) {
    tc::mbar_expect_tx(bar_v, kPanel);
    tc::tma_load_4d(sm + L::kV, &tmV, bar_v, e0, 0, h, b);
    produce_until(kStages, okp);
  }
  int bad = okp ? 0 : 1;
  int cons = 0;  // stage loads consumed so far (same sequence on every thread)
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int t0 = c * kC;
    const int tg = t0 + tid;
    // ---- pass A: S = Qs Ks^T, H = Qs Snap, qn on CUDA cores ------------------------
    float qn = 0.f;
#pragma unroll 1
    for (int pnl = 0; pnl < L::kNP; ++pnl, ++cons) {
      const int slot = cons % kStages;
      if (!tc::mbar_wait(&full[slot], (cons / kStages) & 1, abort_flag)) bad = 1;
      const uint32_t qaddr = sbase + L::kRing + slot * 2 * kPanel;
      if (tid == 0 && !bad) {
        tc::tc_fence_after();
        const uint64_t dq = tc::sdesc_sw128(qaddr, 16, 1024);
        const uint64_t dsn = tc::sdesc_sw128(sbase + L::kSnap + pnl * 4 * 2048, kPanel, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::desc_add(dq, kk * 32);
          tc::mma_bf16(tm + L::tS, ad, tc::desc_add(dq, kPanel + kk * 32), idS, pnl > 0 || kk > 0);
          tc::mma_bf16(tm + L::tH, ad, tc::desc_add(dsn, kk * 2048), idH, pnl > 0 || kk > 0);
        }
        tc::mma_commit(&empty[slot]);
      }
      // qn_t += sum_{j in panel} Qs[t, j] * ns[j]
      {
        const unsigned char* qrow = sm + L::kRing + slot * 2 * kPanel;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 w = *reinterpret_cast<const uint4*>(qrow + tc::sw128_offset(tid, ch * 8));
          const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(x2[e]);
            qn = fmaf(f.x, ns[pnl * 64 + ch * 8 + 2 * e], qn);
            qn = fmaf(f.y, ns[pnl * 64 + ch * 8 + 2 * e + 1], qn);
          }
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[slot]);
      if (tid == 0 && !bad) {
        bool ok = true;
        produce_until(cons + kStages + 1, ok);
        if (!ok) bad = 1;
      }
    }
    if (tid == 0 && !bad) tc::mma_commit(bar_s);
    if (!tc::mbar_wait(bar_v, c & 1, abort_flag)) bad = 1;
    if (!tc::mbar_wait(bar_s, c & 1, abort_flag)) bad = 1;
    tc::tc_fence_after();
    if (__syncthreads_or(bad)) { bad = 1; break; }
    // ---- P = causal(S) -> smem, den_intra ------------------------------------------
    float den_intra = 0.f;
#pragma unroll 1
    for (int s0 = 0; s0 < kC; s0 += 32) {
      float v[32];
      tc::tmem_ld32(tc::taddr(tm, warp * 32, L::tS + s0), v);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = (s0 + j <= tid) ? v[j] : 0.f;
        den_intra += v[j];
      }
      unsigned char* prow = sm + L::kP + (s0 / 64) * kPanel;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack2<__nv_bfloat16>(v[8 * q + 0], v[8 * q + 1]);
        w.y = pack2<__nv_bfloat16>(v[8 * q + 2], v[8 * q + 3]);
        w.z = pack2<__nv_bfloat16>(v[8 * q + 4], v[8 * q + 5]);
        w.w = pack2<__nv_bfloat16>(v[8 * q + 6], v[8 * q + 7]);
        *reinterpret_cast<uint4*>(prow + tc::sw128_offset(tid, (s0 % 64) + 8 * q)) = w;
      }
    }
    // ---- state and n *= decay(c) (per key row = TMEM lane) ---------------------------
    {
      const float* dc = decay + ((int64_t)bh * nch + c) * DK;
#pragma unroll 1
      for (int blk = 0; blk < L::kNB; ++blk) {
        const float dr = dc[blk * 128 + warp * 32 + lane];
#pragma unroll 1
        for (int c0 = 0; c0 < kDV; c0 += 32) {
          float v[32];
          const uint32_t a = tc::taddr(tm, warp * 32, L::tAcc + blk * 64 + c0);
          tc::tmem_ld32(a, v);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= dr;
          tc::tmem_st32(a, v);
        }
        float v[16];  // n blocks are 16 columns apart: touch exactly 16
        const uint32_t a = tc::taddr(tm, warp * 32, L::tN + blk * 16);
        tc::tmem_ld16(a, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] *= dr;
        tc::tmem_st16(a, v);
      }
      tc::tmem_wait_st();
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    if (__syncthreads_or(bad)) { bad = 1; break; }
    // ---- H += P V;  pass B: state += Kh^T V, n += Kh^T 1 ------------------------------------
    if (tid == 0) {
      tc::tc_fence_after();
      const uint64_t dp = tc::sdesc_sw128(sbase + L::kP, 16, 1024);
      const uint64_t dv = tc::sdesc_sw128(sbase + L::kV, kPanel, 1024);
#pragma unroll
      for (int ks = 0; ks < kC / 16; ++ks)
        tc::mma_bf16(tm + L::tH, tc::desc_add(dp, (ks / 4) * kPanel + (ks % 4) * 32), tc::desc_add(dv, ks * 2048),
                     idH, true);
      tc::mma_commit(bar_h);
    }
#pragma unroll 1
    for (int blk = 0; blk < L::kNB; ++blk, ++cons) {
      const int slot = cons % kStages;
      if (!tc::mbar_wait(&full[slot], (cons / kStages) & 1, abort_flag)) bad = 1;
      const uint32_t kaddr = sbase + L::kRing + slot * 2 * kPanel;
      if (tid == 0 && !bad) {
        tc::tc_fence_after();
        const uint64_t dk = tc::sdesc_sw128(kaddr, kPanel, 1024);
        const uint64_t dv = tc::sdesc_sw128(sbase + L::kV, kPanel, 1024);
        const uint64_t d1 = tc::sdesc_sw128(sbase + L::kOnes, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < kC / 16; ++ks) {
          const uint64_t ad = tc::desc_add(dk, ks * 2048);
          tc::mma_bf16(tm + L::tAcc + blk * 64, ad, tc::desc_add(dv, ks * 2048), idAcc, true);
          tc::mma_bf16(tm + L::tN + blk * 16, ad, tc::desc_add(d1, (ks / 4) * 2048 + (ks % 4) * 32), idN, true);
        }
        tc::mma_commit(&empty[slot]);
      }
      if (lane == 0) tc::mbar_arrive(&empty[slot]);
      if (tid == 0 && !bad) {
        bool ok = true;
        produce_until(cons + kStages + 1, ok);
        if (!ok) bad = 1;
      }
    }
    if (tid == 0 && !bad) tc::mma_commit(bar_a);
    if (!tc::mbar_wait(bar_h, c & 1, abort_flag)) bad = 1;
    if (!tc::mbar_wait(bar_a, c & 1, abort_flag)) bad = 1;
    tc::tc_fence_after();
    if (__syncthreads_or(bad)) { bad = 1; break; }
    // next chunk's V (its MMAs are done)
    if (tid == 0 && c + 1 < nch) {
      tc::mbar_expect_tx(bar_v, kPanel);
      tc::tma_load_4d(sm + L::kV, &tmV, bar_v, e0, t0 + kC, h, b);
    }
    // ---- epilogue: h_t = H / max(den, 1) ------------------------------------------------
    {
      const float inv = 1.f / fmaxf(qn + den_intra, 1.f);
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.h) + b * p.sh[0] + h * p.sh[1] + (int64_t)tg * p.th + e0;
#pragma unroll 1
      for (int c0 = 0; c0 < kDV; c0 += 32) {
        float v[32];
        tc::tmem_ld32(tc::taddr(tm, warp * 32, L::tH + c0), v);
        tc::tmem_wait_ld();
        if (tg < p.seqlen && e0 + c0 < p.dv) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<__nv_bfloat16>(v[8 * q + 0] * inv, v[8 * q + 1] * inv);
            w.y = pack2<__nv_bfloat16>(v[8 * q + 2] * inv, v[8 * q + 3] * inv);
            w.z = pack2<__nv_bfloat16>(v[8 * q + 4] * inv, v[8 * q + 5] * inv);
            w.w = pack2<__nv_bfloat16>(v[8 * q + 6] * inv, v[8 * q + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c0 + 8 * q) = w;
          }
        }
      }
    }
    if (c + 1 < nch) snapshot(c + 1);
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
  }

  // ---- final state: true state = TMEM state (m = 0) ----------------------------------------
  if (!bad) {
    tc::tc_fence_after();
#pragma unroll 1
    for (int blk = 0; blk < L::kNB; ++blk) {
      const int row = blk * 128 + warp * 32 + lane;
      if (p.CT) {
#pragma unroll 1
        for (int c0 = 0; c0 < kDV; c0 += 32) {
          float v[32];
          tc::tmem_ld32(tc::taddr(tm, warp * 32, L::tAcc + blk * 64 + c0), v);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (e0 + c0 + j < p.dv) p.CT[((int64_t)bh * DK + row) * p.dv + e0 + c0 + j] = v[j];
        }
      }
      if (p.nT && blockIdx.x == 0) {
        float v[16];
        tc::tmem_ld16(tc::taddr(tm, warp * 32, L::tN + blk * 16), v);
        tc::tmem_wait_ld();
        p.nT[(int64_t)bh * DK + row] = v[0];
      }
    }
    if (p.mT && blockIdx.x == 0 && tid == 0) p.mT[bh] = 0.f;
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tm, 512);
  }
}

// ------------------------------------------------------------------- host --
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t stream_workspace(const Params& p) {
  const size_t nch = (p.seqlen + kC - 1) / kC;
  const size_t ops = (size_t)p.batch * p.heads * p.seqlen * p.dqk * 2;  // bf16 tensor
  const size_t vec = (size_t)p.batch * p.heads * nch * p.dqk * 4;
  return 3 * align256(ops) + 2 * align256(vec);
}

bool stream_shape_ok(const Params& p) {
  if (p.io_dtype != HXM_BF16) return false;
  if (p.dqk != 128 && p.dqk != 256 && p.dqk != 512) return false;
  if (p.dv % 32 != 0 || p.seqlen <= 0) return false;
  auto a16 = [](const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; };
  return a16(p.v) && a16(p.h) && p.sv[0] % 8 == 0 && p.sv[1] % 8 == 0 && p.sh[0] % 8 == 0 && p.sh[1] % 8 == 0 &&
         p.tv % 8 == 0 && p.th % 8 == 0;
}

template <int DK>
static hxm_status launch_stream_dk(const Params& p, cudaStream_t st) {
  using L = SL<DK>;
  if (p.workspace_bytes < stream_workspace(p) || !p.workspace) {
    set_error("hxm_mlstm_chunkwise_fwd: workspace of %zu bytes required (got %zu)", stream_workspace(p),
              p.workspace_bytes);
    return HXM_EBADARG;
  }
  const int nch = (p.seqlen + kC - 1) / kC;
  const size_t ops = align256((size_t)p.batch * p.heads * p.seqlen * DK * 2);
  const size_t vec = align256((size_t)p.batch * p.heads * nch * DK * 4);
  unsigned char* ws = static_cast<unsigned char*>(p.workspace);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(ws);
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(ws + ops);
  __nv_bfloat16* Kh = reinterpret_cast<__nv_bfloat16*>(ws + 2 * ops);
  float* decay = reinterpret_cast<float*>(ws + 3 * ops);
  float* rho_e = reinterpret_cast<float*>(ws + 3 * ops + vec);
  dim3 pg(p.batch * p.heads * nch, (DK + 127) / 128);
  mlstm_prescale_kernel<__nv_bfloat16><<<pg, 128, 0, st>>>(p, Qs, Ks, Kh, decay, rho_e);
  hxm_status s = check_launch("hxm_mlstm_chunkwise_fwd (prescale)");
  if (s != HXM_OK) return s;
  CUtensorMap mq, mk, mh, mv;
  const uint64_t dd[4] = {(uint64_t)DK, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
  const uint64_t sd[3] = {(uint64_t)DK * 2, (uint64_t)p.seqlen * DK * 2, (uint64_t)p.heads * p.seqlen * DK * 2};
  const uint64_t dvd[4] = {(uint64_t)p.dv, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
  const uint64_t sv[3] = {(uint64_t)p.tv * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
  if ((s = make_map_bf16_4d(&mq, Qs, dd, sd, "mlstm Qs")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mk, Ks, dd, sd, "mlstm Ks")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mh, Kh, dd, sd, "mlstm Kh")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mv, p.v, dvd, sv, "mlstm v")) != HXM_OK) return s;
  const size_t smem = L::kBytes + 1024;
  auto kern = mlstm_stream_kernel<DK>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dv + kDV - 1) / kDV, p.heads, p.batch);
  kern<<<grid, 128, smem, st>>>(mq, mk, mh, mv, p, decay, rho_e);
  return check_launch("hxm_mlstm_chunkwise_fwd (stream)");
}

hxm_status launch_stream(const Params& p, cudaStream_t st) {
  if (p.dqk == 128) return launch_stream_dk<128>(p, st);
  if (p.dqk == 256) return launch_stream_dk<256>(p, st);
  return launch_stream_dk<512>(p, st);
}

}  // namespace mlstm
}  // namespace hxm
