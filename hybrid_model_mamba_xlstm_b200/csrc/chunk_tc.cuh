// chunk_tc.cuh — tcgen05 chunkwise linear recurrence with a per-head scalar
// decay: the chunkwise mLSTM ("TFLA", per-head gates) and the Mamba-2 SSD
// chunked scan share this kernel.
//
// Per (batch, head, 64-wide value tile) one CTA walks the sequence in chunks
// of 128 steps.  State S (DK x 64, fp32) lives in TMEM; per chunk
//   b_t = cumsum(log f), u_s = log i_s - b_s, M_t / m the stabilizers:
//   S    = Q K^T                                   (tcgen05, M=N=128)
//   P    = causal(S) * exp(b_t + u_s - M_t)         (threads, bf16 -> smem)
//   Hint = Q . Ssnap     Hintra = P . V            (tcgen05, N=64)
//   qn   = Q . n_snap                              (tcgen05, N=16; mLSTM only)
//   S    = rho * S + (K * kscale)^T V, n likewise   (TMEM rescale + tcgen05)
//   out_t = (sc_t Hint + Hintra) / max(sc_t qn + rowsum P, e^-M_t)   (mLSTM)
//   out_t = e^(b_t) Hint + Hintra + D x_t                              (SSD)
// All exponents are <= 0, so nothing overflows for any gate values; the
// algebra is the reference recurrence (tfla_interface.py:113-137, and the
// Euler scan of scan_interface.py:132-150 for SSD) regrouped by chunk.
//
// Separable weights: with r_t = b_t - M_t, exp(r_t + u_s) = R_t C_s where
// R_t = exp(r_t + c0) and C_s = exp(u_s - c0) for a per-chunk shift c0.  When
// a c0 keeps every R_t and C_s within e^+-40 (checked per chunk on the
// device), P is formed as causal(S) * C_s (one multiply per element, no
// exponential) and R_t is applied to the row's Hintra and rowsum in the
// epilogue; otherwise (a gate range wider than ~e^80 inside one chunk, or the
// ragged last chunk) each element takes its own exponential.
//
// Operands arrive by TMA (128B swizzle) into shared memory; the tensor-core
// operands written by threads (P, the bf16 state snapshot, n) use the same
// swizzled layouts.  One elected thread issues TMA and MMA.  The 8 warps do
// the element-wise work: warp w reads TMEM lanes 32 (w % 4) .. + 31 (one
// chunk row or state row per lane), and the two warps of a lane quarter split
// the columns (half h = w / 4 takes columns 32h .. 32h + 31 of each 64-wide
// block, and of P the 64-column half h).
#pragma once

#include <type_traits>

#include "common.cuh"
#include "tc_sm100.cuh"

namespace hxm {
namespace chunk {

constexpr int kC = 128;      // chunk length (TMEM lanes / MMA M)
constexpr int kDV = 64;      // value columns per CTA
constexpr int kWorkerWarps = 8;                 // element-wise warps
constexpr int kThreads = 32 * kWorkerWarps + 32;  // + one control warp (TMA, MMA)
constexpr int kPanel = 16384;  // one 128-row x 128-byte swizzled panel

enum Mode : int { kMlstm = 0, kSsd = 1 };

struct Params {
  int batch, heads, seqlen, dv;
  // per-step gates, element strides (b, h, t)
  const float* g0;  // mLSTM: log input gate;  SSD: raw dt
  int64_t sg0[3];
  const float* g1;  // mLSTM: log forget gate; SSD: unused
  int64_t sg1[3];
  const float* A;        // SSD: (heads)
  const float* dt_bias;  // SSD: (heads) or null
  int dt_softplus;
  const float* Dskip;    // SSD: (heads) or null
  const __nv_bfloat16* x;  // SSD: x for the D skip, element strides (b, h, t)
  int64_t sx[3];
  __nv_bfloat16* out;    // out[b,h,t,e] element strides (b, h, t), unit e
  int64_t so[3];
  const float* C0;  // (b, h, DK, dv) or SSD (b, h, dv, DK) when state_t
  const float* n0;  // (b, h, DK)
  const float* m0;  // (b, h)
  float* CT;
  float* nT;
  float* mT;
  int state_t;  // state stored transposed (SSD: (b, h, p, n))
  int* error_flag;       // set to 1 when a bounded wait gave up (outputs then unwritten)
  long long wait_limit;  // SM cycles per bounded wait
};

template <int DK>
struct Layout {
  static constexpr int kNB = DK / 128;         // 128-row TMEM blocks of the state
  // Q, K, V of a chunk form one stage; DK = 128 double-buffers them (the next
  // chunk loads, and its S = Q K^T runs, while this chunk finishes)
  static constexpr int kStages = DK == 128 ? 2 : 1;
  static constexpr int kQ = 0;                  // DK/64 panels
  static constexpr int kK = kQ + DK / 64 * kPanel;
  static constexpr int kV = kK + DK / 64 * kPanel;
  static constexpr int kStage = kV + kPanel;    // bytes of one stage
  static constexpr int kP = kStages * kStage;   // 2 panels
  static constexpr int kSnap = kP + 2 * kPanel; // DK rows x 128 B (MN-major, one N panel)
  static constexpr int kN = kSnap + DK * 128;   // n snapshot, K-major [16][DK]: DK/64 panels of 2 KB
  static constexpr int kOnes = kN + DK / 64 * 2048;  // K-major [16][128]: 2 panels of 2 KB
  static constexpr int kMisc = kOnes + 2 * 2048;
  static constexpr int kColW = kMisc;          // float[128]: C_s (separable) or u_s * log2e, by column s
  static constexpr int kDen = kColW + 512;     // float[2][2][128]: rowsum(P) partials of the two column halves, by chunk parity
  static constexpr int kRed = kDen + 2048;     // float[64] reductions
  static constexpr int kBar = kRed + 256;      // 8 x uint64
  static constexpr int kTmemSlot = kBar + 64;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kBytes = kAbort + 12;
  // TMEM columns
  static constexpr int tS = 0, tHint = 128, tHintra = 192, tAcc = 256, tQN = 384, tAccN = 416;
  static_assert(tAcc + 64 * kNB <= tQN, "TMEM layout");
  static_assert(tAccN + 32 * kNB <= 512, "TMEM layout");
};

// Per-row gate values of one chunk, held by the threads of that row.
struct RowGates {
  float r2;  // (b_t - M_t) * log2 e: the per-element exponent's row part (fallback)
  float sc;  // weight of the carried state: exp(b_t + m_in - M_t)
  float R;   // separable row factor exp(b_t - M_t + c0) (1 in the fallback)
  float F;   // normalizer floor exp(-M_t) (mLSTM)
  float ks;  // key scale of row s: exp(g + u_s - m_new)
};

// Named barrier 1 over the 256 element-wise threads (warps 0-7); the control
// warp never takes part.  `_or` returns whether any thread passed v != 0.
HXM_DEV void workers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
HXM_DEV int workers_sync_or(int v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v)
      : "memory");
  return r;
}

template <int DK, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  using Lt = Layout<DK>;
  constexpr bool kNorm = MODE == kMlstm;
  constexpr bool kScaleK = DK == 128;  // key rows scaled (one MMA batch per chunk)
  constexpr int kNP = DK / 64;  // Q/K panels
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled panels
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  float* colw = reinterpret_cast<float*>(sm + Lt::kColW);
  float* denp0 = reinterpret_cast<float*>(sm + Lt::kDen);
  float* red = reinterpret_cast<float*>(sm + Lt::kRed);
  uint64_t* bar_load = reinterpret_cast<uint64_t*>(sm + Lt::kBar);  // TMA: a stage's Q, K, V (one per stage)
  uint64_t* bar_s = bar_load + 2;       // MMA: S done
  uint64_t* bar_a = bar_load + 3;       // MMA: outputs (+ state update, DK = 128) done
  uint64_t* bar_b = bar_load + 4;       // MMA: state update done (DK = 256)
  uint64_t* bar_pready = bar_load + 5;  // workers: P, scaled K, snapshot, decayed state ready
  uint64_t* bar_vready = bar_load + 6;  // workers: scaled V ready (DK = 256)
  uint64_t* bar_fin = bar_load + 7;     // MMA: drain before exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Lt::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + Lt::kAbort);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool worker = warp < kWorkerWarps;
  const int wq = warp & 3;         // TMEM lane quarter
  const int hf = (warp >> 2) & 1;  // column half
  const int row = wq * 32 + lane;  // chunk row t / state row within a 128-row block
  const int ch = 32 * hf;          // this thread's first column of a 64-wide block
  const int e0 = blockIdx.x * kDV;
  const int h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.heads + h;
  const int nchunks = (p.seqlen + kC - 1) / kC;
  const uint32_t sbase = smem_u32(sm);
  const uint32_t tlane = (uint32_t)(wq * 32) << 16;  // this warp's TMEM lane offset

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    tc::mbar_init(bar_load, 1);
    tc::mbar_init(bar_load + 1, 1);
    tc::mbar_init(bar_s, 1);
    tc::mbar_init(bar_a, 1);
    tc::mbar_init(bar_b, 1);
    tc::mbar_init(bar_pready, kWorkerWarps);
    tc::mbar_init(bar_vready, kWorkerWarps);
    tc::mbar_init(bar_fin, 1);
    tc::fence_mbar_init();
    *abort_flag = 0;
    tc::prefetch_tmap(&tmQ);
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
  }
  // ones operand (K-major [16][128]: row 0 = 1) and the n snapshot ([16][DK]: zero)
  {
    uint4* z = reinterpret_cast<uint4*>(sm + Lt::kN);
    for (int i = tid; i < (DK / 64 * 2048 + 2 * 2048) / 16; i += kThreads) z[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    __nv_bfloat16* ones = reinterpret_cast<__nv_bfloat16*>(sm + Lt::kOnes);
    if (tid < 128) {
      const int panel = tid / 64, col = tid % 64;
      ones[(panel * 2048 + tc::sw128_offset(0, col)) / 2] = __float2bfloat16_rn(1.f);
    }
  }
  tc::fence_async_smem();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *tmem_slot + tlane;

  // operand descriptors at the region bases; an MMA adds its byte offset
  const uint64_t dQ = tc::sdesc_sw128(sbase + Lt::kQ, 16, 1024);      // K-major rows t (Q) or s (K)
  const uint64_t dK = tc::sdesc_sw128(sbase + Lt::kK, 16, 1024);
  const uint64_t dKT = tc::sdesc_sw128(sbase + Lt::kK, kPanel, 1024);  // K^T: MN-major, panels = 64 dk rows
  const uint64_t dSnap = tc::sdesc_sw128(sbase + Lt::kSnap, kPanel, 1024);
  const uint64_t dN = tc::sdesc_sw128(sbase + Lt::kN, 16, 1024);
  const uint64_t dP = tc::sdesc_sw128(sbase + Lt::kP, 16, 1024);
  const uint64_t dV = tc::sdesc_sw128(sbase + Lt::kV, kPanel, 1024);
  const uint64_t dOnes = tc::sdesc_sw128(sbase + Lt::kOnes, 16, 1024);
  constexpr uint32_t idS = tc::idesc_bf16(128, 128, false, false);
  constexpr uint32_t idH = tc::idesc_bf16(128, kDV, false, true);
  constexpr uint32_t idQN = tc::idesc_bf16(128, 16, false, false);
  constexpr uint32_t idAcc = tc::idesc_bf16(128, kDV, true, true);
  constexpr uint32_t idAccN = tc::idesc_bf16(128, 16, true, false);

  float m_final = 0.f;  // the stabilizer after the last chunk (workers)
  if (!worker) {
    // ================= control warp: TMA loads and MMAs (one lane) =================
    if (lane == 0) {
      const int hq = (MODE == kSsd) ? 0 : h;
      constexpr uint32_t kLoadBytes = (2 * kNP + 1) * kPanel;
      int waits[2] = {0, 0};     // completed waits per stage barrier (its phase)
      bool pend[2] = {false, false};  // a load issued and not yet waited, per stage
      // Chunk c's operands (stage c % kStages) arrive on the stage's barrier, in
      // one part or in two: Q (free once the output MMAs are done) and K, V
      // (free once the state update is done).
      auto load_q = [&](int c) {
        const int st = c % Lt::kStages;
        tc::mbar_expect_tx(bar_load + st, kLoadBytes);
        pend[st] = true;
        for (int pnl = 0; pnl < kNP; ++pnl)
          tc::tma_load_4d(sm + st * Lt::kStage + Lt::kQ + pnl * kPanel, &tmQ, bar_load + st, pnl * 64, c * kC, hq, b);
      };
      auto load_kv = [&](int c) {
        const int st = c % Lt::kStages;
        for (int pnl = 0; pnl < kNP; ++pnl)
          tc::tma_load_4d(sm + st * Lt::kStage + Lt::kK + pnl * kPanel, &tmK, bar_load + st, pnl * 64, c * kC, hq, b);
        tc::tma_load_4d(sm + st * Lt::kStage + Lt::kV, &tmV, bar_load + st, e0, c * kC, h, b);
      };
      auto wait_load = [&](int c) {
        const int st = c % Lt::kStages;
        const bool ok = tc::mbar_wait(bar_load + st, waits[st] & 1, abort_flag, p.wait_limit);
        if (ok) {
          ++waits[st];
          pend[st] = false;
        }
        return ok;
      };
      const uint32_t tb = *tmem_slot;
      // S = Q K^T of chunk c
      auto issue_s = [&](int c) {
        const uint32_t so = (c % Lt::kStages) * Lt::kStage;
        const uint64_t q = tc::desc_add(dQ, so), k = tc::desc_add(dK, so);
        tc::static_for<DK / 16>([&](auto KS) {
          constexpr int ks = decltype(KS)::value;
          constexpr uint32_t off = (ks / 4) * kPanel + (ks % 4) * 32;
          tc::mma_bf16_at<off, off>(tb + Lt::tS, q, k, idS, ks > 0);
        });
        tc::mma_commit(bar_s);
      };
      // Hint = Q.Snap, qn = Q.n, Hintra = P.V of chunk c
      auto issue_out = [&](int c) {
        const uint32_t so = (c % Lt::kStages) * Lt::kStage;
        const uint64_t q = tc::desc_add(dQ, so), v = tc::desc_add(dV, so);
        tc::static_for<DK / 16>([&](auto KS) {
          constexpr int ks = decltype(KS)::value;
          constexpr uint32_t qoff = (ks / 4) * kPanel + (ks % 4) * 32;
          tc::mma_bf16_at<qoff, ks * 2048>(tb + Lt::tHint, q, dSnap, idH, ks > 0);
          if (kNorm) tc::mma_bf16_at<qoff, (ks / 4) * 2048 + (ks % 4) * 32>(tb + Lt::tQN, q, dN, idQN, ks > 0);
        });
        tc::static_for<kC / 16>([&](auto KS) {
          constexpr int ks = decltype(KS)::value;
          tc::mma_bf16_at<(ks / 4) * kPanel + (ks % 4) * 32, ks * 2048>(tb + Lt::tHintra, dP, v, idH, ks > 0);
        });
      };
      // state update of chunk c (A = K^T: M = 128 state rows = K panels 2blk,
      // 2blk+1 (LBO = panel stride); K step = 16 rows); the normalizer's B row
      // 0 is 1 (K scaled) or kscale (V scaled)
      auto issue_update = [&](int c) {
        const uint32_t so = (c % Lt::kStages) * Lt::kStage;
        const uint64_t kt = tc::desc_add(dKT, so), v = tc::desc_add(dV, so);
        tc::static_for<Lt::kNB * (kC / 16)>([&](auto I) {
          constexpr int blk = decltype(I)::value / (kC / 16), ks = decltype(I)::value % (kC / 16);
          constexpr uint32_t aoff = (2 * blk) * kPanel + ks * 2048;
          tc::mma_bf16_at<aoff, ks * 2048>(tb + Lt::tAcc + blk * 64, kt, v, idAcc, true);
          if (kNorm)
            tc::mma_bf16_at<aoff, (ks / 4) * 2048 + (ks % 4) * 32>(tb + Lt::tAccN + blk * 32, kt, dOnes, idAccN, true);
        });
      };
      load_q(0);
      load_kv(0);
      if (Lt::kStages == 2 && nchunks > 1) {
        load_q(1);
        load_kv(1);
      }
      bool ok = wait_load(0);
      if (ok) {
        tc::tc_fence_after();
        issue_s(0);
      }
#pragma unroll 1
      for (int c = 0; ok && c < nchunks; ++c) {
        if (!tc::mbar_wait(bar_pready, c & 1, abort_flag, p.wait_limit)) break;
        tc::tc_fence_after();
        issue_out(c);
        if (kScaleK) {
          issue_update(c);
          tc::mma_commit(bar_a);
          // the next chunk's S right behind (its stage loaded a chunk ahead)
          if (c + 1 < nchunks) {
            if (!wait_load(c + 1)) break;
            tc::tc_fence_after();
            issue_s(c + 1);
          }
          if (!tc::mbar_wait(bar_a, c & 1, abort_flag, p.wait_limit)) break;
          if (c + 2 < nchunks) {  // this chunk's stage is free
            load_q(c + 2);
            load_kv(c + 2);
          }
        } else {
          tc::mma_commit(bar_a);
          if (!tc::mbar_wait(bar_a, c & 1, abort_flag, p.wait_limit)) break;
          if (c + 1 < nchunks) load_q(c + 1);
          if (!tc::mbar_wait(bar_vready, c & 1, abort_flag, p.wait_limit)) break;
          tc::tc_fence_after();
          issue_update(c);
          tc::mma_commit(bar_b);
          if (!tc::mbar_wait(bar_b, c & 1, abort_flag, p.wait_limit)) break;
          if (c + 1 < nchunks) {
            load_kv(c + 1);
            if (!wait_load(c + 1)) break;
            tc::tc_fence_after();
            issue_s(c + 1);
          }
        }
      }
      // Leave nothing in flight: every MMA of this thread done, and (after a
      // wait that gave up) the loads issued and not waited landed — all bounded.
      volatile int no_abort = 0;
      tc::mma_commit(bar_fin);
      tc::mbar_wait(bar_fin, 0, &no_abort, 20000000ll);
      for (int st = 0; st < Lt::kStages; ++st)
        if (pend[st]) tc::mbar_wait(bar_load + st, waits[st] & 1, &no_abort, 20000000ll);
    }
    __syncwarp();
  } else {
    // ================= workers: gates, P, scaling, epilogue, snapshots =================
    const float A_h = (MODE == kSsd) ? p.A[h] : 0.f;
    const float dtb = (MODE == kSsd && p.dt_bias) ? p.dt_bias[h] : 0.f;
    const float Dh = (MODE == kSsd && p.Dskip) ? p.Dskip[h] : 0.f;

    // ---- initial state -> TMEM (fp32) ----------------------------------------
    float m_prev = (kNorm && p.m0) ? p.m0[bh] : 0.f;
#pragma unroll 1
    for (int blk = 0; blk < Lt::kNB; ++blk) {
      const int srow = blk * 128 + row;  // state row (dk index)
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = e0 + ch + j;
        float x = 0.f;
        if (p.C0 && col < p.dv)
          x = p.state_t ? p.C0[((int64_t)bh * p.dv + col) * DK + srow] : p.C0[((int64_t)bh * DK + srow) * p.dv + col];
        v[j] = x;
      }
      tc::tmem_st32(tm + Lt::tAcc + blk * 64 + ch, v);
      if (hf == 1) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        if (kNorm && p.n0) v[0] = p.n0[(int64_t)bh * DK + srow];
        tc::tmem_st32(tm + Lt::tAccN + blk * 32, v);
      }
    }
    tc::tmem_wait_st();

    // state (TMEM fp32) -> bf16 snapshots in shared memory, then the state is
    // decayed in place by the next chunk's rho (one TMEM pass for both)
    auto snapshot = [&](float rho) {
#pragma unroll 1
      for (int blk = 0; blk < Lt::kNB; ++blk) {
        const int srow = blk * 128 + row;
        unsigned char* sp = sm + Lt::kSnap;
        float v[32];
        const uint32_t a = tm + Lt::tAcc + blk * 64 + ch;
        tc::tmem_ld32(a, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack2<__nv_bfloat16>(v[8 * q + 0], v[8 * q + 1]);
          w.y = pack2<__nv_bfloat16>(v[8 * q + 2], v[8 * q + 3]);
          w.z = pack2<__nv_bfloat16>(v[8 * q + 4], v[8 * q + 5]);
          w.w = pack2<__nv_bfloat16>(v[8 * q + 6], v[8 * q + 7]);
          *reinterpret_cast<uint4*>(sp + tc::sw128_offset(srow, ch + 8 * q)) = w;
        }
        if (rho != 1.f) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= rho;
          tc::tmem_st32(a, v);
        }
        if (kNorm && hf == 1) {
          const uint32_t an = tm + Lt::tAccN + blk * 32;
          const float n = tc::tmem_ld1(an);
          tc::tmem_wait_ld();
          __nv_bfloat16* nb =
              reinterpret_cast<__nv_bfloat16*>(sm + Lt::kN + (srow / 64) * 2048 + tc::sw128_offset(0, srow % 64));
          *nb = __float2bfloat16_rn(n);
          if (rho != 1.f) tc::tmem_st1(an, n * rho);
        }
      }
      tc::tmem_wait_st();
    };

    // This row's raw gate inputs of chunk cc (global loads, issued a chunk
    // ahead of their use): mLSTM log i, log f; SSD raw dt.
    auto load_gates = [&](int cc, float& x0, float& x1) {
      const int tgc = cc * kC + row;
      x0 = 0.f;
      x1 = 0.f;
      if (tgc < p.seqlen) {
        x0 = p.g0[b * p.sg0[0] + h * p.sg0[1] + (int64_t)tgc * p.sg0[2]];
        if (MODE == kMlstm) x1 = p.g1[b * p.sg1[0] + h * p.sg1[1] + (int64_t)tgc * p.sg1[2]];
      }
    };
    // Gates of chunk cc: b_t = cumsum log f, u_s, the stabilizers M_t / m_new
    // (from m_in, the state's scale entering the chunk), the state's decay rho,
    // this row's RowGates, whether the weights separate, and the column vector
    // colw (C_s, or u_s * log2e).  Every thread takes part (two barriers); colw
    // is written after the caller's last read of the previous chunk's values.
    auto compute_gates = [&](int cc, float x0, float x1, float m_in, RowGates& rg, float& rho_out, float& m_out,
                             bool& sep_out) {
      const bool v = cc * kC + row < p.seqlen;
      float li, lf;
      if (MODE == kMlstm) {
        li = v ? x0 : -INFINITY;
        lf = v ? x1 : 0.f;
      } else {
        float dtv = v ? x0 + dtb : 0.f;
        if (p.dt_softplus) dtv = (dtv > 20.f) ? dtv : log1pf(__expf(dtv));
        li = (v && dtv > 0.f) ? __logf(dtv) : -INFINITY;
        lf = v ? dtv * A_h : 0.f;
      }
      // pass 1: b_t = inclusive sum of log f over the rows, g = the chunk total
      float bt = lf;
  #pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, bt, o);
        if (lane >= o) bt += n;
      }
      if (lane == 31) red[hf * 4 + wq] = bt;
      workers_sync();
      float g = 0.f;
  #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = red[hf * 4 + i];
        if (i < wq) bt += x;
        g += x;
      }
      const float us = li - bt;
      // pass 2: prefix max of u (mLSTM), extremes of u (and of b, SSD), u_0
      float pm = us, umin = us, bmax = bt, bmin = bt;
      if (kNorm) {
  #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float n = __shfl_up_sync(0xffffffffu, pm, o);
          if (lane >= o) pm = fmaxf(pm, n);
        }
      } else {
  #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
          bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
          bmin = fminf(bmin, __shfl_xor_sync(0xffffffffu, bmin, o));
        }
      }
  #pragma unroll
      for (int o = 16; o > 0; o >>= 1) umin = fminf(umin, __shfl_xor_sync(0xffffffffu, umin, o));
      if (lane == 31) {
        red[8 + hf * 4 + wq] = pm;  // the warp's max of u
        red[16 + hf * 4 + wq] = umin;
        red[24 + hf * 4 + wq] = bmax;
        red[32 + hf * 4 + wq] = bmin;
      }
      if (row == 0) red[40 + hf] = us;
      workers_sync();
      float U = -INFINITY, umn = INFINITY, bmx = -INFINITY, bmn = INFINITY, pre = -INFINITY;
  #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = red[8 + hf * 4 + i];
        if (i < wq) pre = fmaxf(pre, x);
        U = fmaxf(U, x);
        umn = fminf(umn, red[16 + hf * 4 + i]);
        bmx = fmaxf(bmx, red[24 + hf * 4 + i]);
        bmn = fminf(bmn, red[32 + hf * 4 + i]);
      }
      float rt, m_new, rmax, rmin;
      if (kNorm) {
        const float mx = fmaxf(m_in, fmaxf(pm, pre));  // max(m_in, prefix max of u)
        const float Mt = bt + mx;
        m_new = g + fmaxf(m_in, U);
        rt = -mx;  // b_t - M_t, nonincreasing in t
        rmax = -fmaxf(m_in, red[40 + hf]);
        rmin = -fmaxf(m_in, U);
        rg.sc = __expf(m_in - mx);
        rg.F = __expf(-Mt);
      } else {
        m_new = 0.f;
        rt = bt;
        rmax = bmx;
        rmin = bmn;
        rg.sc = __expf(bt);
        rg.F = 0.f;
      }
      rg.ks = __expf(g + us - m_new);
      rg.r2 = rt * kLog2e;
      rho_out = __expf(g + m_in - m_new);
      m_out = m_new;
      // a shift c0 with every rt + c0 and us - c0 inside [-40, 40]?
      const float lo = fmaxf(-rmin - 40.f, U - 40.f);
      const float hi = fminf(40.f - rmax, 40.f + umn);
      const bool sep = lo <= hi;  // false for any non-finite extreme (e.g. a row past the end)
      const float c0 = 0.5f * (lo + hi);
      rg.R = sep ? __expf(rt + c0) : 1.f;
      if (hf == 0) colw[row] = sep ? __expf(us - c0) : us * kLog2e;
      sep_out = sep;
    };

    RowGates gc;
    float rho_cur, m_new_cur;
    bool sep_cur;
    float gx0, gx1;  // the next chunk's raw gate inputs
    load_gates(0, gx0, gx1);
    compute_gates(0, gx0, gx1, m_prev, gc, rho_cur, m_new_cur, sep_cur);
    if (nchunks > 1) load_gates(1, gx0, gx1);
    snapshot(rho_cur);
    workers_sync();  // colw of chunk 0 written
    tc::fence_async_smem();
    tc::tc_fence_before();

    int bad = 0;
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
      const int t0 = c * kC;
      const int tg = t0 + row;
      const bool valid = tg < p.seqlen;
      float* denp = denp0 + (c & 1) * 2 * kC;
      // ---- wait S; P = causal(S) * weight -> smem (bf16), this half's 64 columns ----
      if (!tc::mbar_wait(bar_s, c & 1, abort_flag, p.wait_limit)) bad = 1;
      tc::tc_fence_after();
      {
        float2 den2 = make_float2(0.f, 0.f);  // rowsum of P, two partial sums
        unsigned char* pp = sm + Lt::kP + hf * kPanel;
        auto block = [&](int sb) {
          const int s0 = 64 * hf + 32 * sb;
          float v[32];
          const bool need = s0 <= wq * 32 + 31;
          if (need) {
            tc::tmem_ld32(tm + Lt::tS + s0, v);
            tc::tmem_wait_ld();
            const float4* cw = reinterpret_cast<const float4*>(colw + s0);
            // DIAG: the block on the diagonal (s0 = 32 (warp % 4)), where column
            // s0 + j is causal for this row iff j <= lane; blocks left of it are all causal
            auto weigh = [&](auto diag_tag, auto sep_tag) {
              constexpr bool kDiag = decltype(diag_tag)::value;
              constexpr bool kSep = decltype(sep_tag)::value;
  #pragma unroll
              for (int j4 = 0; j4 < 8; ++j4) {
                const float4 c4 = cw[j4];
  #pragma unroll
                for (int k = 0; k < 2; ++k) {
                  const int j = 4 * j4 + 2 * k;
                  float2 w = k ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
                  if (!kSep) {
                    w = __fadd2_rn(make_float2(gc.r2, gc.r2), w);
                    w = make_float2(ex2_approx(w.x), ex2_approx(w.y));
                  }
                  float2 pv = __fmul2_rn(make_float2(v[j], v[j + 1]), w);
                  if (kDiag) {
                    if (j > lane) pv.x = 0.f;
                    if (j + 1 > lane) pv.y = 0.f;
                  }
                  v[j] = pv.x;
                  v[j + 1] = pv.y;
                  den2 = __fadd2_rn(den2, pv);
                }
              }
            };
            if (s0 == wq * 32) {
              if (sep_cur) weigh(std::true_type{}, std::true_type{});
              else weigh(std::true_type{}, std::false_type{});
            } else {
              if (sep_cur) weigh(std::false_type{}, std::true_type{});
              else weigh(std::false_type{}, std::false_type{});
            }
          } else {
  #pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
  #pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<__nv_bfloat16>(v[8 * q + 0], v[8 * q + 1]);
            w.y = pack2<__nv_bfloat16>(v[8 * q + 2], v[8 * q + 3]);
            w.z = pack2<__nv_bfloat16>(v[8 * q + 4], v[8 * q + 5]);
            w.w = pack2<__nv_bfloat16>(v[8 * q + 6], v[8 * q + 7]);
            *reinterpret_cast<uint4*>(pp + tc::sw128_offset(row, 32 * sb + 8 * q)) = w;
          }
        };
        block(0);
        block(1);
        denp[hf * kC + row] = den2.x + den2.y;
      }
      // ---- kscale (row s = this thread's row): DK = 128 scales the K rows here
      //      (this half's dk panel), so that one MMA batch below does the outputs
      //      and the state update, (kscale . K)^T V; DK = 256 scales the V rows
      //      after the output MMAs (half the elements of a K row).
      if (kScaleK) {
        const float ks = gc.ks;
        unsigned char* krow = sm + (c % Lt::kStages) * Lt::kStage + Lt::kK + hf * kPanel;
  #pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4* ptr = reinterpret_cast<uint4*>(krow + tc::sw128_offset(row, 8 * q));
          uint4 w = *ptr;
          uint32_t* e = reinterpret_cast<uint32_t*>(&w);
  #pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __fmul2_rn(__bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&e[j])), make_float2(ks, ks));
            e[j] = pack2<__nv_bfloat16>(f.x, f.y);
          }
          *ptr = w;
        }
      }
      // SSD D skip: this row's x values from the staged V (= x) panel
      uint4 xrow[4];
      if (MODE == kSsd) {
  #pragma unroll
        for (int q = 0; q < 4; ++q)
          xrow[q] = *reinterpret_cast<const uint4*>(sm + (c % Lt::kStages) * Lt::kStage + Lt::kV +
                                                    tc::sw128_offset(row, ch + 8 * q));
      }
      // ---- P, scaled K, the snapshot and the decayed state are ready ----------------
      tc::fence_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_pready);
      // next chunk's gates while the tensor core works on this chunk
      RowGates gn = gc;
      float rho_next = 1.f, m_new_next = m_new_cur;
      bool sep_next = sep_cur;
      if (c + 1 < nchunks) {
        compute_gates(c + 1, gx0, gx1, m_new_cur, gn, rho_next, m_new_next, sep_next);
        if (c + 2 < nchunks) load_gates(c + 2, gx0, gx1);
      }
      if (!tc::mbar_wait(bar_a, c & 1, abort_flag, p.wait_limit)) bad = 1;
      tc::tc_fence_after();
      if (!kScaleK) {
        // V rows *= kscale, the normalizer's B row 0 = kscale: the update is K^T (kscale . V)
        const float ks = gc.ks;
        unsigned char* vrow = sm + Lt::kV;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4* ptr = reinterpret_cast<uint4*>(vrow + tc::sw128_offset(row, ch + 8 * q));
          uint4 w = *ptr;
          uint32_t* e = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __fmul2_rn(__bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&e[j])), make_float2(ks, ks));
            e[j] = pack2<__nv_bfloat16>(f.x, f.y);
          }
          *ptr = w;
        }
        if (kNorm && hf == 0) {
          __nv_bfloat16* kv = reinterpret_cast<__nv_bfloat16*>(sm + Lt::kOnes);
          kv[((row / 64) * 2048 + tc::sw128_offset(0, row % 64)) / 2] = __float2bfloat16_rn(ks);
        }
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_vready);
      }
      // every worker agrees to go on (and the rowsum partials of P are visible)
      if (workers_sync_or(bad)) { bad = 1; break; }
      // ---- epilogue: output row t, this half's 32 columns ---------------------------
      {
        const float den_intra = denp[row] + denp[kC + row];
        float o[32];
        {
          float hi[32], ha[32];
          tc::tmem_ld32(tm + Lt::tHint + ch, hi);
          tc::tmem_ld32(tm + Lt::tHintra + ch, ha);
          const float qn = kNorm ? tc::tmem_ld1(tm + Lt::tQN) : 0.f;
          tc::tmem_wait_ld();
          if (kNorm) {
            const float den = fmaxf(gc.sc * qn + gc.R * den_intra, gc.F);
            const float inv = 1.f / den;
            const float a = gc.sc * inv, r = gc.R * inv;
  #pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = fmaf(a, hi[j], r * ha[j]);
          } else {
  #pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = fmaf(gc.sc, hi[j], gc.R * ha[j]);
          }
        }
        const bool ok = valid && e0 + ch < p.dv;
        if (MODE == kSsd && ok && Dh != 0.f) {
  #pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w = xrow[q];
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&w);
  #pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(x2[j]);
              o[8 * q + 2 * j] = fmaf(Dh, f.x, o[8 * q + 2 * j]);
              o[8 * q + 2 * j + 1] = fmaf(Dh, f.y, o[8 * q + 2 * j + 1]);
            }
          }
        }
        if (ok) {
          __nv_bfloat16* orow = p.out + b * p.so[0] + h * p.so[1] + (int64_t)tg * p.so[2] + e0 + ch;
  #pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<__nv_bfloat16>(o[8 * q + 0], o[8 * q + 1]);
            w.y = pack2<__nv_bfloat16>(o[8 * q + 2], o[8 * q + 3]);
            w.z = pack2<__nv_bfloat16>(o[8 * q + 4], o[8 * q + 5]);
            w.w = pack2<__nv_bfloat16>(o[8 * q + 6], o[8 * q + 7]);
            *reinterpret_cast<uint4*>(orow + 8 * q) = w;
          }
        }
      }
      if (!kScaleK) {
        if (!tc::mbar_wait(bar_b, c & 1, abort_flag, p.wait_limit)) bad = 1;
        tc::tc_fence_after();
      }
      // ---- snapshot of the updated state for the next chunk's Hint, decayed state ----
      snapshot(rho_next);
      m_prev = m_new_cur;
      m_new_cur = m_new_next;
      gc = gn;
      sep_cur = sep_next;
      tc::fence_async_smem();
      tc::tc_fence_before();
    }
    m_final = m_prev;
  }

  // ---- final state (none after a wait that gave up: every give-up raised the
  //      abort flag, read by all threads after the barrier) ------------------------
  tc::tc_fence_before();
  __syncthreads();
  const bool ok = *abort_flag == 0;
  if (worker && ok) {
    tc::tc_fence_after();
#pragma unroll 1
    for (int blk = 0; blk < Lt::kNB; ++blk) {
      const int srow = blk * 128 + row;
      if (p.CT) {
        float v[32];
        tc::tmem_ld32(tm + Lt::tAcc + blk * 64 + ch, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = e0 + ch + j;
          if (col < p.dv) {
            if (p.state_t) p.CT[((int64_t)bh * p.dv + col) * DK + srow] = v[j];
            else p.CT[((int64_t)bh * DK + srow) * p.dv + col] = v[j];
          }
        }
      }
      if (kNorm && p.nT && blockIdx.x == 0 && hf == 1) {
        const float n = tc::tmem_ld1(tm + Lt::tAccN + blk * 32);
        tc::tmem_wait_ld();
        p.nT[(int64_t)bh * DK + srow] = n;
      }
    }
    if (kNorm && p.mT && blockIdx.x == 0 && tid == 0) p.mT[bh] = m_final;
  } else if (!ok && tid == 0) {
    if (p.error_flag) atomicExch(p.error_flag, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(*tmem_slot, 512);
  }
}

}  // namespace chunk
}  // namespace hxm
