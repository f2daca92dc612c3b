// mlstm_stream.cu — chunkwise mLSTM on tcgen05 for per-channel gates and for
// dqk up to 512, streaming the key dimension through shared memory.
//
// Two kernels:
//  1. mlstm_prescale_kernel (CUDA cores, one pass over q, k, gates): per chunk
//     of 128 steps and key channel j, with b_t[j] = sum_{s<=t} log f_s[j] inside
//     the chunk, g[j] = b_127[j] and the midpoint rho[j] = g[j] / 2:
//        Qs[t,j] = q[t,j] e^(b_t - rho)              (|exponent| <= |g|/2)
//        Ks[s,j] = k[s,j] e^(rho - b_s + log i_s)
//        decay[j] = e^g,  rho_e[j] = e^rho,  nadd[j] = sum_s Ks[s,j] e^rho
//     so that  sum_j q_t k_s e^(b_t - b_s + log i_s) = Qs_t . Ks_s  (intra-chunk)
//     and      state' = diag(e^g) state + diag(e^rho) Ks^T v   (inter-chunk),
//     the recurrence of tfla_forward_pytorch (tfla_interface.py:113-137) with
//     gates multiplying along the key dimension (mlstm_block.py:117-129).
//  2. mlstm_stream_kernel (tcgen05): per (b, h, 64-wide value tile), per chunk
//        S  = Qs Ks^T, H = Qs (rho_e . state) + causal(S) V     (TMEM)
//        qn = Qs (rho_e . n) on CUDA cores,  den = qn + rowsum(causal S)
//        h  = H / max(den, 1)
//        state = decay . state + rho_e . Ks^T V,  n = decay . n + nadd
//     TMEM keeps the state divided by the current chunk's rho_e per key row,
//     so the update adds plain Ks^T V from the same Ks panels as S, and the
//     per-row factors rho_e(c-1), rho_e(c) (snapshot and decay at once) are
//     applied when the state is read back for the next chunk.  Two 64-channel
//     key panels (Qs and Ks of each) per 64 KB slot stream through a 2-slot
//     TMA ring; n lives in shared memory.
//  Range: every factor above is e^x with |x| <= |g|/2 + |log i|.  The
//  prescale pass checks each exponent it forms against +-kMaxExp and flags
//  the (b, h) pair when one is outside or not finite: a chunk whose forget
//  gates sum below about -160 per channel, input gates beyond e^+-75 or so,
//  f = 0.  The stream kernel skips flagged pairs and the exact recurrent
//  kernel (mlstm_recurrent.cu) runs them in the same call, so the results
//  hold for any gate values the reference itself computes without overflow.
//  kMaxExp = 80: fp32 / bf16 hold e^+-87; one chunk adds at most
//  sum_s e^80 |k_s||v_s| to the stored state (below 3.4e38 while that sum of
//  |k||v| over the chunk's 128 steps stays below 6e3, e.g. RMS-normalized k),
//  and the snapshot e^rho C of a state entry stays a normal bf16 down to 7e-4
//  (smaller entries of a state carry a share of q.C below bf16 rounding).
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
constexpr float kMaxExp = 80.f;  // largest |exponent| of a chunk factor the stream kernel takes

// ---------------------------------------------------------------- pre-pass --
// grid (B*H*nchunks, ceil(DK/(128*NJ))), block 128: thread = NJ adjacent key
// channels (NJ = 2: bf16x2 loads and stores, 128 bytes per warp access).
// Per-head gates: the factors e^(b_t - rho), e^(rho - b_t + log i_t) are the
// same for every channel, so the block forms them once per step (thread t,
// one scan over the chunk) and the channels only multiply; per-channel gates
// take two exponentials per element.
// Chunks of kc steps (128, or 64 for the pairs a 128-step pass flagged).  unsafe[b*heads + h]
// is raised to level + 1 when an exponent is beyond +-kMaxExp or not finite; with level 1 only
// the pairs flagged by the level-0 pass are processed (the rest of the grid returns at once).
// fqg != NULL (per-head gates, raw-q mode): the per-step query factors e^(b_t - rho) go to
// fqg[b*heads + h][t] instead of into a scaled copy of q; Qs is neither read nor written.
template <typename T, int NJ>
__global__ void __launch_bounds__(128) mlstm_prescale_kernel(const Params p, __nv_bfloat16* Qs, __nv_bfloat16* Ks,
                                                             float* decay, float* rho_e, float* nadd, int* unsafe,
                                                             int kc, int level, float* fqg) {
  __shared__ float fq[kC], fk[kC], red[4];
  const int nch = (p.seqlen + kc - 1) / kc;
  const int c = blockIdx.x % nch;
  const int bh = blockIdx.x / nch;
  if (level > 0 && unsafe[bh] == 0) return;  // uniform over the block
  const int b = bh / p.heads, h = bh % p.heads;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int j0 = (blockIdx.y * 128 + tid) * NJ;
  const bool active = j0 < p.dqk;  // every thread takes part in the block scan below
  const int t0 = c * kc, tn = min(kc, p.seqlen - t0);
  const T* q = static_cast<const T*>(p.q) + b * p.sq[0] + h * p.sq[1];
  const T* k = static_cast<const T*>(p.k) + b * p.sk[0] + h * p.sk[1];
  const float* li = p.log_i + b * p.si[0] + h * p.si[1];
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1];
  const bool pc = p.gate_mode == 1;  // uniform over the grid
  float g[NJ];
  if (!pc) {
    // per-step factors of the chunk: thread t holds step t
    const float lft = tid < tn ? lf[(int64_t)(t0 + tid) * p.tf] : 0.f;
    const float lit = tid < tn ? li[(int64_t)(t0 + tid) * p.ti] : 0.f;
    float bt = lft;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, bt, o);
      if (lane >= o) bt += n;
    }
    if (lane == 31) red[w] = bt;
    __syncthreads();
    float gs = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i < w) bt += red[i];
      gs += red[i];
    }
    const float rho = 0.5f * gs;
    const float xq = bt - rho, xk = rho - bt + lit;
    // !(x <= max) also catches NaN (e.g. log f = -inf); one store per flagged block suffices
    if (!(fabsf(xq) <= kMaxExp) || !(fabsf(xk) <= kMaxExp)) unsafe[bh] = level + 1;
    fq[tid] = __expf(xq);
    fk[tid] = __expf(xk);
    if (fqg && blockIdx.y == 0 && tid < tn) fqg[(int64_t)bh * p.seqlen + t0 + tid] = fq[tid];
    __syncthreads();
#pragma unroll
    for (int u = 0; u < NJ; ++u) g[u] = gs;
  } else {
#pragma unroll
    for (int u = 0; u < NJ; ++u) g[u] = 0.f;
    if (active) {
#pragma unroll 4
      for (int t = 0; t < tn; ++t) {
#pragma unroll
        for (int u = 0; u < NJ; ++u) g[u] += lf[(int64_t)(t0 + t) * p.tf + j0 + u];
      }
    }
  }
  if (!active) return;  // no barrier below
  float bt[NJ], ksum[NJ], eh[NJ];
#pragma unroll
  for (int u = 0; u < NJ; ++u) {
    bt[u] = ksum[u] = 0.f;
    eh[u] = __expf(0.5f * g[u]);  // e^rho
  }
  const int64_t ob = (int64_t)bh * p.seqlen * p.dqk;
  bool bad = false;
#pragma unroll 4
  for (int t = 0; t < tn; ++t) {
    const int64_t tt = t0 + t;
    float qv[NJ] = {}, kv[NJ];
    if (NJ == 2) {
      const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162*>(k + tt * p.tk + j0);
      const float2 kf = __bfloat1622float2(k2);
      kv[0] = kf.x; kv[NJ - 1] = kf.y;
      if (!fqg) {
        const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q + tt * p.tq + j0));
        qv[0] = qf.x; qv[NJ - 1] = qf.y;
      }
    } else {
      kv[0] = to_f32<T>(k[tt * p.tk + j0]);
      if (!fqg) qv[0] = to_f32<T>(q[tt * p.tq + j0]);
    }
    float qs[NJ], ks[NJ], kh[NJ];
#pragma unroll
    for (int u = 0; u < NJ; ++u) {
      float a, e;
      if (!pc) {
        a = fq[t];
        e = fk[t];
      } else {
        bt[u] += lf[tt * p.tf + j0 + u];
        const float rho = 0.5f * g[u];
        const float xq = bt[u] - rho, xk = rho - bt[u] + li[tt * p.ti + j0 + u];
        bad |= !(fabsf(xq) <= kMaxExp) || !(fabsf(xk) <= kMaxExp);
        a = __expf(xq);
        e = __expf(xk);
      }
      qs[u] = qv[u] * a;
      ks[u] = kv[u] * e;
      kh[u] = ks[u] * eh[u];
      ksum[u] += kh[u];
    }
    const int64_t o = ob + tt * p.dqk + j0;
    if (NJ == 2) {
      if (!fqg) *reinterpret_cast<uint32_t*>(Qs + o) = pack2<__nv_bfloat16>(qs[0], qs[NJ - 1]);
      *reinterpret_cast<uint32_t*>(Ks + o) = pack2<__nv_bfloat16>(ks[0], ks[NJ - 1]);
    } else {
      if (!fqg) Qs[o] = __float2bfloat16_rn(qs[0]);
      Ks[o] = __float2bfloat16_rn(ks[0]);
    }
  }
  if (bad) unsafe[bh] = level + 1;
#pragma unroll
  for (int u = 0; u < NJ; ++u) {
    const int64_t vi = ((int64_t)bh * nch + c) * p.dqk + j0 + u;
    decay[vi] = __expf(g[u]);
    rho_e[vi] = eh[u];
    nadd[vi] = ksum[u];  // e^rho Ks^T 1: the normalizer's increment
  }
}

// Per-channel gates, two channels per thread (4-byte q, k accesses): the same outputs as the
// per-channel branch of mlstm_prescale_kernel, with the chunk's steps split over 8 segments
// (one warp each) instead of walked by one thread: block = 32 channel pairs x 8 segments.
// Each thread sums its segment's log forget gates, the segments' sums are scanned through
// shared memory, and each thread then forms its segment's factors from that prefix — so a
// thread's serial chain is kc / 8 steps, and a small call (one sequence, four heads, one
// 128-step chunk: 8 blocks of the one-thread-per-channel kernel, 140 us) spreads over 32 blocks
// of 256 threads.  Warp accesses per step: 256 contiguous bytes of each gate row, 128 of q, k.
constexpr int kPcSeg = 8;
__global__ void __launch_bounds__(32 * kPcSeg) mlstm_prescale_channels_kernel(
    const Params p, __nv_bfloat16* Qs, __nv_bfloat16* Ks, float* decay, float* rho_e, float* nadd, int* unsafe,
    int kc, int level) {
  __shared__ float2 part[kPcSeg][32];
  const int nch = (p.seqlen + kc - 1) / kc;
  const int c = blockIdx.x % nch;
  const int bh = blockIdx.x / nch;
  if (level > 0 && unsafe[bh] == 0) return;  // uniform over the block
  const int b = bh / p.heads, h = bh % p.heads;
  const int cp = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int j0 = blockIdx.y * 64 + 2 * cp;
  const bool active = j0 < p.dqk;  // every thread takes part in the barriers below
  const int t0 = c * kc, tn = min(kc, p.seqlen - t0);
  const int sl = kc / kPcSeg, ta = min(seg * sl, tn), te = min(ta + sl, tn);
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q) + b * p.sq[0] + h * p.sq[1];
  const __nv_bfloat16* k = static_cast<const __nv_bfloat16*>(p.k) + b * p.sk[0] + h * p.sk[1];
  const float* li = p.log_i + b * p.si[0] + h * p.si[1] + j0;
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1] + j0;
  float2 s = make_float2(0.f, 0.f);
  if (active) {
#pragma unroll 4
    for (int t = ta; t < te; ++t) {
      const int64_t tt = t0 + t;
      s.x += lf[tt * p.tf];
      s.y += lf[tt * p.tf + 1];
    }
  }
  part[seg][cp] = s;
  __syncthreads();
  float2 pre = make_float2(0.f, 0.f), g = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kPcSeg; ++i) {
    const float2 v = part[i][cp];
    if (i < seg) pre = make_float2(pre.x + v.x, pre.y + v.y);
    g = make_float2(g.x + v.x, g.y + v.y);
  }
  const float rho[2] = {0.5f * g.x, 0.5f * g.y};
  const float eh[2] = {__expf(rho[0]), __expf(rho[1])};
  float bt[2] = {pre.x, pre.y}, ksum[2] = {0.f, 0.f};
  bool bad = false;
  const int64_t ob = (int64_t)bh * p.seqlen * p.dqk;
  if (active) {
#pragma unroll 4
    for (int t = ta; t < te; ++t) {
      const int64_t tt = t0 + t;
      const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(k + tt * p.tk + j0));
      const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q + tt * p.tq + j0));
      const float kv[2] = {kf.x, kf.y}, qv[2] = {qf.x, qf.y};
      float qs[2], ks[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        bt[u] += lf[tt * p.tf + u];
        const float xq = bt[u] - rho[u], xk = rho[u] - bt[u] + li[tt * p.ti + u];
        bad |= !(fabsf(xq) <= kMaxExp) || !(fabsf(xk) <= kMaxExp);  // also catches NaN
        qs[u] = qv[u] * __expf(xq);
        ks[u] = kv[u] * __expf(xk);
        ksum[u] += ks[u] * eh[u];
      }
      const int64_t o = ob + tt * p.dqk + j0;
      *reinterpret_cast<uint32_t*>(Qs + o) = pack2<__nv_bfloat16>(qs[0], qs[1]);
      *reinterpret_cast<uint32_t*>(Ks + o) = pack2<__nv_bfloat16>(ks[0], ks[1]);
    }
  }
  if (bad) unsafe[bh] = level + 1;
  __syncthreads();  // every thread has read part[] above
  part[seg][cp] = make_float2(ksum[0], ksum[1]);
  __syncthreads();
  if (seg == 0 && active) {
    float2 tot = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kPcSeg; ++i) tot = make_float2(tot.x + part[i][cp].x, tot.y + part[i][cp].y);
    const int64_t vi = ((int64_t)bh * nch + c) * p.dqk + j0;
    decay[vi] = __expf(g.x);
    decay[vi + 1] = __expf(g.y);
    rho_e[vi] = eh[0];
    rho_e[vi + 1] = eh[1];
    nadd[vi] = tot.x;  // e^rho Ks^T 1: the normalizer's increment
    nadd[vi + 1] = tot.y;
  }
}

// Per-head gates with 16-byte-aligned k (and q) rows: the same outputs as the per-head branch
// of mlstm_prescale_kernel, one block per (b, h, chunk) over every key channel, each thread
// moving 8 channels (16 bytes) of one step per access — the other kernel's 4-byte accesses left
// it latency-bound at about 1.5 TB/s.  Threads 0..kc-1 first scan the chunk's log forget gates
// (one step each) into the per-step factors.
constexpr int kPreThreads = 256;
template <int DK>
__global__ void __launch_bounds__(kPreThreads) mlstm_prescale_heads_kernel(
    const Params p, __nv_bfloat16* Qs, __nv_bfloat16* Ks, float* decay, float* rho_e, float* nadd, int* unsafe,
    int kc, int level, float* fqg) {
  constexpr int kOct = DK / 8;                 // 16-byte groups of a key row
  constexpr int kRows = kPreThreads / kOct;    // steps handled in parallel
  __shared__ float fq[kC], fk[kC], red[8];
  __shared__ float ksum_s[kRows][DK];
  const int nch = (p.seqlen + kc - 1) / kc;
  const int c = blockIdx.x % nch;
  const int bh = blockIdx.x / nch;
  if (level > 0 && unsafe[bh] == 0) return;  // uniform over the block
  const int b = bh / p.heads, h = bh % p.heads;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int t0 = c * kc, tn = min(kc, p.seqlen - t0);
  const float* li = p.log_i + b * p.si[0] + h * p.si[1];
  const float* lf = p.log_f + b * p.sf[0] + h * p.sf[1];
  // per-step factors: thread t holds step t (warps 0-3), prefix sums by shuffles + 4 partials
  float bt = 0.f, lit = 0.f;
  if (tid < kC) {
    bt = tid < tn ? lf[(int64_t)(t0 + tid) * p.tf] : 0.f;
    lit = tid < tn ? li[(int64_t)(t0 + tid) * p.ti] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, bt, o);
      if (lane >= o) bt += n;
    }
    if (lane == 31) red[w] = bt;
  }
  __syncthreads();
  float gs = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (tid < kC && i < w) bt += red[i];
    gs += red[i];
  }
  const float rho = 0.5f * gs;
  if (tid < kC) {
    const float xq = bt - rho, xk = rho - bt + lit;
    if (!(fabsf(xq) <= kMaxExp) || !(fabsf(xk) <= kMaxExp)) unsafe[bh] = level + 1;
    fq[tid] = __expf(xq);
    fk[tid] = __expf(xk);
    if (fqg && tid < tn) fqg[(int64_t)bh * p.seqlen + t0 + tid] = fq[tid];
  }
  __syncthreads();
  const float eh = __expf(rho);
  const int oct = tid % kOct, r0 = tid / kOct, j0 = oct * 8;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q) + b * p.sq[0] + h * p.sq[1] + j0;
  const __nv_bfloat16* k = static_cast<const __nv_bfloat16*>(p.k) + b * p.sk[0] + h * p.sk[1] + j0;
  const int64_t ob = (int64_t)bh * p.seqlen * DK + j0;
  float ks8[8] = {};
#pragma unroll 4
  for (int t = r0; t < tn; t += kRows) {
    const int64_t tt = t0 + t;
    const uint4 kw = *reinterpret_cast<const uint4*>(k + tt * p.tk);
    const float e = fk[t];
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kw);
    uint4 ko;
    uint32_t* kop = reinterpret_cast<uint32_t*>(&ko);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 kf = __bfloat1622float2(k2[i]);
      const float a = kf.x * e, bb = kf.y * e;
      ks8[2 * i] += a;
      ks8[2 * i + 1] += bb;
      kop[i] = pack2<__nv_bfloat16>(a, bb);
    }
    *reinterpret_cast<uint4*>(Ks + ob + tt * DK) = ko;
    if (!fqg) {
      const uint4 qw = *reinterpret_cast<const uint4*>(q + tt * p.tq);
      const float f = fq[t];
      const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qw);
      uint4 qo;
      uint32_t* qop = reinterpret_cast<uint32_t*>(&qo);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 qf = __bfloat1622float2(q2[i]);
        qop[i] = pack2<__nv_bfloat16>(qf.x * f, qf.y * f);
      }
      *reinterpret_cast<uint4*>(Qs + ob + tt * DK) = qo;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) ksum_s[r0][j0 + i] = ks8[i];
  __syncthreads();
  for (int j = tid; j < DK; j += kPreThreads) {
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kRows; ++r) sum += ksum_s[r][j];
    const int64_t vi = ((int64_t)bh * nch + c) * DK + j;
    decay[vi] = __expf(gs);
    rho_e[vi] = eh;
    nadd[vi] = eh * sum;  // e^rho Ks^T 1: the normalizer's increment
  }
}

// ------------------------------------------------------------ stream kernel --
// Warps 0-7: element-wise work (warp w reads TMEM lanes 32 (w % 4) .., the two
// warps of a lane quarter split the columns: half h = w / 4).  Warp 8: the
// MMA issuer (and the V loads).  Warp 9: the TMA producer of the Q/K panel ring.
constexpr int kWorkers = 8;
constexpr int kStreamThreads = 32 * kWorkers + 64;

template <int DK>
struct SL {
  static constexpr int kNP = DK / 64;                 // key panels
  static constexpr int kNB = DK / 128;                // state row blocks (TMEM 128 lanes)
  // a ring slot holds the Qs and Ks panels of two consecutive 64-channel key
  // panels, [Qs 2i | Ks 2i | Qs 2i+1 | Ks 2i+1]: the S and Qs.Snap MMAs of both
  // and the state update of block i (its 128 key rows = the two Ks panels) read it
  static constexpr int kLPC = (DK + 127) / 128;       // ring loads per chunk
  static constexpr int kSlotB = 4 * kPanel;           // bytes per slot
  // P lives inside the snapshot buffer when that is large enough (the
  // snapshot is consumed by the chunk's Qs.Snap MMAs before P is written, and
  // rewritten only after P.V is done)
  static constexpr bool kPinSnap = DK >= 256;
  static constexpr int kStages = 2;
  static constexpr int kRing = 0;                     // kStages x 64 KB
  static constexpr int kSnap = kRing + kStages * kSlotB;  // DK rows x 128 B (MN-major B, one 64-wide N panel)
  static constexpr int kP = kPinSnap ? kSnap : kSnap + DK * 128;  // 2 panels
  static constexpr int kV = kPinSnap ? kSnap + DK * 128 : kP + 2 * kPanel;  // 1 panel
  static constexpr int kN = kV + kPanel;              // float [DK]  n, the normalizer state
  static constexpr int kNs = kN + DK * 4;             // float [DK]  rho_e . n   (for qn)
  static constexpr int kRow = kNs + DK * 4;           // float [2 parity][2 (qn, rowsum)][2 half][128]
  static constexpr int kBar = kRow + 2 * 2 * 2 * 128 * 4;  // full[kStages], empty[kStages], v, s, pready, b, snap, fin
  static constexpr int kSlot = kBar + 8 * (2 * kStages + 6);
  static constexpr int kAbort = kSlot + 4;
  static constexpr int kBytes = kAbort + 12;
  // TMEM columns: S 0..127, H (double buffered) 128..255, state blocks 256 + 64 b
  static constexpr int tS = 0, tH = 128, tAcc = 256;
  static_assert(tAcc + 64 * kNB <= 512, "TMEM layout");
};

// Named barrier 1 over the 256 element-wise threads; `_or`: any thread's v != 0.
HXM_DEV void stream_workers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
HXM_DEV int stream_workers_sync_or(int v) {
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

template <int DK>
__global__ void __launch_bounds__(kStreamThreads, 1)
    mlstm_stream_kernel(const __grid_constant__ CUtensorMap tmQs, const __grid_constant__ CUtensorMap tmKs,
                        const __grid_constant__ CUtensorMap tmV,
                        const Params p, const float* __restrict__ decay, const float* __restrict__ rho_e,
                        const float* __restrict__ nadd, const int* __restrict__ unsafe, int kc, int want,
                        const float* __restrict__ fqg) {
  // this launch runs the pairs whose range level is `want` (0: 128-step chunks, 1: 64-step
  // chunks); the others belong to another launch (uniform over the CTA)
  if (unsafe[blockIdx.z * p.heads + blockIdx.y] != want) return;
  using L = SL<DK>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint64_t* empty = full + L::kStages;
  uint64_t* bar_v = empty + L::kStages;  // TMA: V of the chunk
  uint64_t* bar_s = bar_v + 1;        // MMA: S and Qs.Snap of the chunk
  uint64_t* bar_pready = bar_v + 2;   // workers: P written
  uint64_t* bar_b = bar_v + 3;        // MMA: P.V and the state update
  uint64_t* bar_snap = bar_v + 4;     // workers: snapshot, decayed state; the older H buffer read
  uint64_t* bar_fin = bar_v + 5;      // MMA: drain before exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::kSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::kAbort);
  float* nst = reinterpret_cast<float*>(sm + L::kN);
  float* ns = reinterpret_cast<float*>(sm + L::kNs);
  float* rowv = reinterpret_cast<float*>(sm + L::kRow);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wq = warp & 3, hf = (warp >> 2) & 1;
  const int row = wq * 32 + lane;  // chunk row t / state row within a 128-row block
  const int ch = 32 * hf;
  const int e0 = blockIdx.x * kDV, h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.heads + h;
  const int nch = (p.seqlen + kc - 1) / kc;
  const uint32_t sbase = smem_u32(sm);
  // 64-step chunks load 64-row boxes into the upper half of each 128-row operand panel; the
  // lower half stays zero (zeroed here), so every MMA keeps its 128-row shape and the extra
  // rows contribute nothing
  const uint32_t slot_bytes = kc == kC ? L::kSlotB : L::kSlotB / 2;
  const uint32_t v_bytes = kc == kC ? kPanel : kPanel / 2;

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    for (int i = 0; i < L::kStages; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1 + kWorkers);  // MMA commit + one arrive per worker warp
    }
    tc::mbar_init(bar_v, 1);
    tc::mbar_init(bar_s, 1);
    tc::mbar_init(bar_pready, kWorkers);
    tc::mbar_init(bar_b, 1);
    tc::mbar_init(bar_snap, kWorkers);
    tc::mbar_init(bar_fin, 1);
    tc::fence_mbar_init();
    *abort_flag = 0;
  }
  if (!L::kPinSnap) {  // P: blocks right of the diagonal are never written again
    uint4* zp = reinterpret_cast<uint4*>(sm + L::kP);
    for (int i = tid; i < 2 * kPanel / 16; i += kStreamThreads) zp[i] = make_uint4(0, 0, 0, 0);
  }
  if (kc != kC) {  // the ring's and V's rows past the chunk: zero for the whole launch
    uint4* zr = reinterpret_cast<uint4*>(sm + L::kRing);
    for (int i = tid; i < L::kStages * L::kSlotB / 16; i += kStreamThreads) zr[i] = make_uint4(0, 0, 0, 0);
    uint4* zv = reinterpret_cast<uint4*>(sm + L::kV);
    for (int i = tid; i < kPanel / 16; i += kStreamThreads) zv[i] = make_uint4(0, 0, 0, 0);
  }
  tc::fence_async_smem();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = *tmem_slot;
  const uint32_t tm = tb + ((uint32_t)(wq * 32) << 16);
  const uint64_t dSnap = tc::sdesc_sw128(sbase + L::kSnap, kPanel, 1024);
  const uint64_t dP = tc::sdesc_sw128(sbase + L::kP, 16, 1024);
  const uint64_t dV = tc::sdesc_sw128(sbase + L::kV, kPanel, 1024);
  constexpr uint32_t idS = tc::idesc_bf16(128, 128, false, false);
  constexpr uint32_t idH = tc::idesc_bf16(128, kDV, false, true);
  constexpr uint32_t idAcc = tc::idesc_bf16(128, kDV, true, true);
  const int total_loads = nch * L::kLPC;

  if (warp == kWorkers) {
    // ================= MMA issuer (one lane) =================
    if (lane == 0) {
      int loads_v = 0, waited_v = 0;
      auto load_v = [&](int c) {
        tc::mbar_expect_tx(bar_v, v_bytes);
        tc::tma_load_4d(sm + L::kV, &tmV, bar_v, e0, c * kc, h, b);
        ++loads_v;
      };
      load_v(0);
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const uint32_t tH = tb + L::tH + (c & 1) * kDV;
        if (!tc::mbar_wait(bar_snap, c & 1, abort_flag, p.wait_limit)) break;
        tc::tc_fence_after();
        // the state update below needs this chunk's V
        if (!tc::mbar_wait(bar_v, waited_v & 1, abort_flag, p.wait_limit)) break;
        ++waited_v;
        tc::tc_fence_after();
        // S = Qs Ks^T, H = Qs Snap and state += Ks^T V, slot by slot from the ring
        bool ok = true;
#pragma unroll 1
        for (int i = 0; i < L::kLPC; ++i) {
          const int idx = c * L::kLPC + i, slot = idx % L::kStages;
          if (!tc::mbar_wait(&full[slot], (idx / L::kStages) & 1, abort_flag, p.wait_limit)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t sb = sbase + L::kRing + slot * L::kSlotB;
#pragma unroll
          for (int pp = 0; pp < 2; ++pp) {
            const int pnl = 2 * i + pp;
            const uint64_t dq = tc::sdesc_sw128(sb + pp * 2 * kPanel, 16, 1024);
            const uint64_t dsn = tc::desc_add(dSnap, pnl * 4 * 2048);
            const bool acc = pnl > 0;
            tc::static_for<4>([&](auto KK) {
              constexpr int kk = decltype(KK)::value;
              tc::mma_bf16_at<kk * 32, kPanel + kk * 32>(tb + L::tS, dq, dq, idS, acc || kk > 0);
              tc::mma_bf16_at<kk * 32, kk * 2048>(tH, dq, dsn, idH, acc || kk > 0);
            });
          }
          if (i + 1 == L::kLPC) tc::mma_commit(bar_s);
          // block i: A = Ks^T (MN-major, the two Ks panels 2 panels apart)
          const uint64_t dk = tc::sdesc_sw128(sb + kPanel, 2 * kPanel, 1024);
          const uint32_t tAcc = tb + L::tAcc + i * 64;
          tc::static_for<kC / 16>([&](auto KS) {
            constexpr int ks = decltype(KS)::value;
            tc::mma_bf16_at<ks * 2048, ks * 2048>(tAcc, dk, dV, idAcc, true);
          });
          tc::mma_commit(&empty[slot]);
        }
        if (!ok) break;
        // H += P V once P is written
        if (!tc::mbar_wait(bar_pready, c & 1, abort_flag, p.wait_limit)) break;
        tc::tc_fence_after();
        tc::static_for<kC / 16>([&](auto KS) {
          constexpr int ks = decltype(KS)::value;
          tc::mma_bf16_at<(ks / 4) * kPanel + (ks % 4) * 32, ks * 2048>(tH, dP, dV, idH, true);
        });
        tc::mma_commit(bar_b);
        if (!tc::mbar_wait(bar_b, c & 1, abort_flag, p.wait_limit)) break;
        if (c + 1 < nch) load_v(c + 1);  // V is free
      }
      // leave nothing in flight (bounded): the MMAs, and a V load not waited for
      volatile int no_abort = 0;
      tc::mma_commit(bar_fin);
      tc::mbar_wait(bar_fin, 0, &no_abort, 20000000ll);
      if (loads_v > waited_v) tc::mbar_wait(bar_v, waited_v & 1, &no_abort, 20000000ll);
    }
    __syncwarp();
  } else if (warp == kWorkers + 1) {
    // ================= TMA producer of the panel ring (one lane) =================
    if (lane == 0) {
      int issued = 0;
#pragma unroll 1
      for (int idx = 0; idx < total_loads; ++idx) {
        const int slot = idx % L::kStages;
        if (idx >= L::kStages && !tc::mbar_wait(&empty[slot], ((idx / L::kStages) - 1) & 1, abort_flag, p.wait_limit)) break;
        const int c = idx / L::kLPC, i = idx % L::kLPC;
        unsigned char* dst = sm + L::kRing + slot * L::kSlotB;
        tc::mbar_expect_tx(&full[slot], slot_bytes);
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          const int pnl = 2 * i + pp;
          tc::tma_load_4d(dst + pp * 2 * kPanel, &tmQs, &full[slot], pnl * 64, c * kc, h, b);
          tc::tma_load_4d(dst + pp * 2 * kPanel + kPanel, &tmKs, &full[slot], pnl * 64, c * kc, h, b);
        }
        ++issued;
      }
      // after a give-up: the last kStages loads issued land before exit (bounded)
      if (*abort_flag) {
        volatile int no_abort = 0;
        for (int idx = issued - L::kStages; idx < issued; ++idx)
          if (idx >= 0) tc::mbar_wait(&full[idx % L::kStages], (idx / L::kStages) & 1, &no_abort, 20000000ll);
      }
    }
    __syncwarp();
  } else {
    // ================= workers =================
    // initial state -> TMEM (the caller's stabilized C0 / n0 scaled by e^m0), n -> smem
    const float s0 = p.m0 ? __expf(p.m0[bh]) : 1.f;
#pragma unroll 1
    for (int blk = 0; blk < L::kNB; ++blk) {
      const int srow = blk * 128 + row;
      float v[32];
      const float* crow = p.C0 ? p.C0 + ((int64_t)bh * DK + srow) * p.dv + e0 + ch : nullptr;
      if (crow && e0 + ch + 32 <= p.dv && p.dv % 4 == 0 && reinterpret_cast<uintptr_t>(p.C0) % 16 == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {  // the row's 128 bytes in 16-byte loads
          const float4 c4 = *reinterpret_cast<const float4*>(crow + j);
          v[j] = s0 * c4.x; v[j + 1] = s0 * c4.y; v[j + 2] = s0 * c4.z; v[j + 3] = s0 * c4.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (crow && e0 + ch + j < p.dv) ? s0 * crow[j] : 0.f;
      }
      tc::tmem_st32(tm + L::tAcc + blk * 64 + ch, v);
    }
    for (int j = tid; j < DK; j += 32 * kWorkers) nst[j] = p.n0 ? s0 * p.n0[(int64_t)bh * DK + j] : 0.f;
    tc::tmem_wait_st();
    stream_workers_sync();

    // Entering chunk c (after the update of chunk c-1): the bf16 snapshot
    // rho_e(c) . state for Qs Snap, the state decayed in place by decay(c) (one
    // TMEM pass), ns = rho_e(c) . n and n = decay(c) . n + nadd(c).
    // This thread's per-chunk vectors: rho_e, decay of its state rows (one per
    // block) and of its normalizer entries j = tid, tid + 256; loaded a chunk
    // ahead of their use.
    constexpr int kNJ = (DK + 32 * kWorkers - 1) / (32 * kWorkers);
    // fp, fc: the per-row factors rho_e(c-1), rho_e(c) of the state pass below
    struct ChunkVec {
      float fp[L::kNB], fc[L::kNB], nre[kNJ], ndc[kNJ], nad[kNJ];
    };
    auto load_vec = [&](int c, ChunkVec& cv) {
      const int64_t vo = ((int64_t)bh * nch + c) * DK;
#pragma unroll
      for (int blk = 0; blk < L::kNB; ++blk) {
        cv.fc[blk] = rho_e[vo + blk * 128 + row];
        cv.fp[blk] = c > 0 ? rho_e[vo - DK + blk * 128 + row] : 1.f;
      }
#pragma unroll
      for (int i = 0; i < kNJ; ++i) {
        const int j = tid + i * 32 * kWorkers;
        cv.nre[i] = j < DK ? rho_e[vo + j] : 0.f;
        cv.ndc[i] = j < DK ? decay[vo + j] : 0.f;
        cv.nad[i] = j < DK ? nadd[vo + j] : 0.f;
      }
    };
    // TMEM holds the state divided by the current chunk's e^(g/2) per key row
    // (the update adds Ks^T V, rho_e^-1 of the true increment); entering chunk c, the
    // factors rho_e(c-1) (back to the true state) then rho_e(c) per row both form the
    // snapshot rho_e(c) . state and decay the stored state for chunk c.  Applied one
    // after the other: their product alone falls below the fp32 normal range once the
    // two chunks' log forget gates sum below about -175, while each partial result
    // stays in range.
    auto snapshot = [&](const ChunkVec& cv) {
      // state blocks two at a time (both TMEM loads in flight before the wait)
      auto block = [&](int blk, float (&v)[32]) {
        const int srow = blk * 128 + row;
        const float fp = cv.fp[blk], fc = cv.fc[blk];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 t2 = __fmul2_rn(make_float2(v[j], v[j + 1]), make_float2(fp, fp));
          const float2 d2 = __fmul2_rn(t2, make_float2(fc, fc));
          v[j] = d2.x;
          v[j + 1] = d2.y;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack2<__nv_bfloat16>(v[8 * q + 0], v[8 * q + 1]);
          w.y = pack2<__nv_bfloat16>(v[8 * q + 2], v[8 * q + 3]);
          w.z = pack2<__nv_bfloat16>(v[8 * q + 4], v[8 * q + 5]);
          w.w = pack2<__nv_bfloat16>(v[8 * q + 6], v[8 * q + 7]);
          *reinterpret_cast<uint4*>(sm + L::kSnap + tc::sw128_offset(srow, ch + 8 * q)) = w;
        }
        tc::tmem_st32(tm + L::tAcc + blk * 64 + ch, v);
      };
      if constexpr (L::kNB == 1) {
        float v[32];
        tc::tmem_ld32(tm + L::tAcc + ch, v);
        tc::tmem_wait_ld();
        block(0, v);
      } else {
#pragma unroll
        for (int blk = 0; blk < L::kNB; blk += 2) {
          float v0[32], v1[32];
          tc::tmem_ld32(tm + L::tAcc + blk * 64 + ch, v0);
          tc::tmem_ld32(tm + L::tAcc + (blk + 1) * 64 + ch, v1);
          tc::tmem_wait_ld();
          block(blk, v0);
          block(blk + 1, v1);
        }
      }
#pragma unroll
      for (int i = 0; i < kNJ; ++i) {
        const int j = tid + i * 32 * kWorkers;
        if (j < DK) {
          const float n = nst[j];
          ns[j] = cv.nre[i] * n;
          nst[j] = cv.ndc[i] * n + cv.nad[i];
        }
      }
      tc::tmem_wait_st();
      tc::fence_async_smem();
      tc::tc_fence_before();
    };
    ChunkVec cvn;  // the next snapshot's vectors
    load_vec(0, cvn);
    snapshot(cvn);
    if (nch > 1) load_vec(1, cvn);
    stream_workers_sync();  // ns of chunk 0 written
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar_snap);

    // Output rows of chunk c: h_t = H / max(qn + rowsum, 1), this half's 32
    // columns, from H buffer c & 1 (the next chunk's Qs.Snap runs into the other).
    // Raw-q mode (fqg): H, qn and the row sum were formed with q itself, so the
    // step's query factor f_t scales them here: h_t = f_t H / max(f_t (qn + rowsum), 1).
    auto epilogue = [&](int c) {
      {
        const int tg = c * kc + row;
        const float* qnp = rowv + (c & 1) * 512;
        const float* denp = qnp + 256;
        const float fr = (fqg && row < kc && tg < p.seqlen) ? fqg[(int64_t)bh * p.seqlen + tg] : 1.f;
        const float inv = fr / fmaxf(fr * (qnp[row] + qnp[kC + row] + denp[row] + denp[kC + row]), 1.f);
        float v[32];
        tc::tmem_ld32(tm + L::tH + (c & 1) * kDV + ch, v);
        tc::tmem_wait_ld();
        if (row < kc && tg < p.seqlen && e0 + ch < p.dv) {
          __nv_bfloat16* orow =
              static_cast<__nv_bfloat16*>(p.h) + b * p.sh[0] + h * p.sh[1] + (int64_t)tg * p.th + e0 + ch;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack2<__nv_bfloat16>(v[8 * q + 0] * inv, v[8 * q + 1] * inv);
            w.y = pack2<__nv_bfloat16>(v[8 * q + 2] * inv, v[8 * q + 3] * inv);
            w.z = pack2<__nv_bfloat16>(v[8 * q + 4] * inv, v[8 * q + 5] * inv);
            w.w = pack2<__nv_bfloat16>(v[8 * q + 6] * inv, v[8 * q + 7] * inv);
            *reinterpret_cast<uint4*>(orow + 8 * q) = w;
          }
        }
        tc::tc_fence_before();
      }
    };
    int bad = 0;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      float* qnp = rowv + (c & 1) * 512;  // [2 half][128]
      float* denp = qnp + 256;            // [2 half][128]
      // ---- pass A: this half's panels' qn_t partial = Qs[t, panel] . ns[panel] ---------
      float qn = 0.f;
#pragma unroll 1
      for (int i = 0; i < L::kLPC; ++i) {
        const int idx = c * L::kLPC + i, slot = idx % L::kStages;
        if (!tc::mbar_wait(&full[slot], (idx / L::kStages) & 1, abort_flag, p.wait_limit)) bad = 1;
        {  // this half's panel of the slot: 2i + hf
          const int pnl = 2 * i + hf;
          const unsigned char* qrow = sm + L::kRing + slot * L::kSlotB + hf * 2 * kPanel;
          const float4* n4 = reinterpret_cast<const float4*>(ns + pnl * 64);
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 w = *reinterpret_cast<const uint4*>(qrow + tc::sw128_offset(row, q * 8));
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&w);
            const float4 na = n4[2 * q], nb = n4[2 * q + 1];
            acc = __ffma2_rn(__bfloat1622float2(x2[0]), make_float2(na.x, na.y), acc);
            acc = __ffma2_rn(__bfloat1622float2(x2[1]), make_float2(na.z, na.w), acc);
            acc = __ffma2_rn(__bfloat1622float2(x2[2]), make_float2(nb.x, nb.y), acc);
            acc = __ffma2_rn(__bfloat1622float2(x2[3]), make_float2(nb.z, nb.w), acc);
          }
          qn += acc.x + acc.y;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[slot]);
        // the previous chunk's outputs leave while this chunk's later panels load
        if (i == (L::kLPC + 1) / 2 - 1 && c > 0) epilogue(c - 1);
      }
      qnp[hf * kC + row] = qn;
      // ---- P = causal(S) -> smem (bf16), this half's 64 columns; rowsum partial --------
      if (!tc::mbar_wait(bar_s, c & 1, abort_flag, p.wait_limit)) bad = 1;
      tc::tc_fence_after();
      {
        float2 den2 = make_float2(0.f, 0.f);
        unsigned char* pp = sm + L::kP + hf * kPanel;
#pragma unroll 1
        for (int sb = 0; sb < 2; ++sb) {
          const int s0 = 64 * hf + 32 * sb;
          float v[32];
          if (s0 > wq * 32 + 31) {  // warp-uniform: right of the diagonal
            if (!L::kPinSnap) continue;  // stays zero from the start
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(pp + tc::sw128_offset(row, 32 * sb + 8 * q)) = make_uint4(0, 0, 0, 0);
            continue;
          }
          tc::tmem_ld32(tm + L::tS + s0, v);
          tc::tmem_wait_ld();
          const bool diag = s0 == wq * 32;  // column s0 + j causal for this row iff j <= lane
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float2 pv = make_float2(v[j], v[j + 1]);
            if (diag) {
              if (j > lane) pv.x = 0.f;
              if (j + 1 > lane) pv.y = 0.f;
            }
            v[j] = pv.x;
            v[j + 1] = pv.y;
            den2 = __fadd2_rn(den2, pv);
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
        }
        denp[hf * kC + row] = den2.x + den2.y;
      }
      tc::fence_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_pready);
      if (!tc::mbar_wait(bar_b, c & 1, abort_flag, p.wait_limit)) bad = 1;
      tc::tc_fence_after();
      // every worker agrees to go on (the qn / rowsum partials are visible)
      if (stream_workers_sync_or(bad)) { bad = 1; break; }
      // ---- the next chunk's snapshot; its Qs . Snap may start while this chunk's
      //      outputs leave from the other H buffer ---------------------------------------
      if (c + 1 < nch) {
        snapshot(cvn);
        if (c + 2 < nch) load_vec(c + 2, cvn);
        stream_workers_sync();  // ns of chunk c + 1 written
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_snap);
      }
    }
    if (!bad) epilogue(nch - 1);
  }

  // ---- final state (none after a wait that gave up) ------------------------------------
  tc::tc_fence_before();
  __syncthreads();
  const bool ok = *abort_flag == 0;
  if (warp < kWorkers && ok) {
    tc::tc_fence_after();
#pragma unroll 1
    for (int blk = 0; blk < L::kNB; ++blk) {
      const int srow = blk * 128 + row;
      if (p.CT) {
        // the stored state times the last chunk's rho_e
        const float rl = rho_e[((int64_t)bh * nch + nch - 1) * DK + srow];
        float v[32];
        tc::tmem_ld32(tm + L::tAcc + blk * 64 + ch, v);
        tc::tmem_wait_ld();
        float* crow = p.CT + ((int64_t)bh * DK + srow) * p.dv + e0 + ch;
        if (e0 + ch + 32 <= p.dv && p.dv % 4 == 0 && reinterpret_cast<uintptr_t>(p.CT) % 16 == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(crow + j) = make_float4(rl * v[j], rl * v[j + 1], rl * v[j + 2], rl * v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (e0 + ch + j < p.dv) crow[j] = rl * v[j];
        }
      }
    }
    if (p.nT && blockIdx.x == 0)
      for (int j = tid; j < DK; j += 32 * kWorkers) p.nT[(int64_t)bh * DK + j] = nst[j];
    if (p.mT && blockIdx.x == 0 && tid == 0) p.mT[bh] = 0.f;
  } else if (!ok && tid == 0 && p.error_flag) {
    atomicExch(p.error_flag, 1);  // a bounded wait gave up: this tile's outputs are not written
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tb, 512);
  }
}

// ------------------------------------------------------------------- host --
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t stream_workspace(const Params& p) {
  const size_t nch = (p.seqlen + kC / 2 - 1) / (kC / 2);  // per-chunk vectors sized for 64-step chunks
  const size_t ops = (size_t)p.batch * p.heads * p.seqlen * p.dqk * 2;  // bf16 tensor
  const size_t vec = (size_t)p.batch * p.heads * nch * p.dqk * 4;
  const size_t flags = (size_t)p.batch * p.heads * 4;  // per (b, h): out of the kernel's range
  const size_t fq = (size_t)p.batch * p.heads * p.seqlen * 4;  // per-step query factors (raw-q mode)
  return 2 * align256(ops) + 3 * align256(vec) + align256(flags) + align256(fq);
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
  const int nch64 = (p.seqlen + kC / 2 - 1) / (kC / 2);
  const size_t ops = align256((size_t)p.batch * p.heads * p.seqlen * DK * 2);
  const size_t vec = align256((size_t)p.batch * p.heads * nch64 * DK * 4);
  unsigned char* ws = static_cast<unsigned char*>(p.workspace);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(ws);
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(ws + ops);
  float* decay = reinterpret_cast<float*>(ws + 2 * ops);
  float* rho_e = reinterpret_cast<float*>(ws + 2 * ops + vec);
  float* nadd = reinterpret_cast<float*>(ws + 2 * ops + 2 * vec);
  int* unsafe = reinterpret_cast<int*>(ws + 2 * ops + 3 * vec);
  float* fq = reinterpret_cast<float*>(ws + 2 * ops + 3 * vec + align256((size_t)p.batch * p.heads * 4));
  HXM_CUDA_TRY(cudaMemsetAsync(unsafe, 0, sizeof(int) * (size_t)p.batch * p.heads, st));
  // Per-head gates: the query factor is one scalar per step, so the tensor cores take q itself
  // (TMA straight from the caller's tensor) and the epilogue applies the factor per row; the
  // prescale pass then neither reads q nor writes a scaled copy of it.
  const bool raw_q = p.gate_mode == 0 && reinterpret_cast<uintptr_t>(p.q) % 16 == 0 && p.tq % 8 == 0 &&
                     p.sq[0] % 8 == 0 && p.sq[1] % 8 == 0;
  float* fqg = raw_q ? fq : nullptr;
  // two channels per thread when q, k rows allow 4-byte loads
  const bool pair = p.tq % 2 == 0 && p.tk % 2 == 0 && p.sq[0] % 2 == 0 && p.sq[1] % 2 == 0 && p.sk[0] % 2 == 0 &&
                    p.sk[1] % 2 == 0 && reinterpret_cast<uintptr_t>(p.q) % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(p.k) % 4 == 0;
  // per-head gates with 16-byte-aligned k (and, unless raw-q, q) rows: the vectorized pass
  auto rows16 = [](const void* x, int64_t t, const int64_t* sx) {
    return reinterpret_cast<uintptr_t>(x) % 16 == 0 && t % 8 == 0 && sx[0] % 8 == 0 && sx[1] % 8 == 0;
  };
  const bool heads16 = p.gate_mode == 0 && rows16(p.k, p.tk, p.sk) && (raw_q || rows16(p.q, p.tq, p.sq));
  auto prescale = [&](int kc, int level) {
    const int nch = (p.seqlen + kc - 1) / kc;
    if (heads16) {
      mlstm_prescale_heads_kernel<DK><<<p.batch * p.heads * nch, kPreThreads, 0, st>>>(
          p, Qs, Ks, decay, rho_e, nadd, unsafe, kc, level, fqg);
    } else if (pair && p.gate_mode == 1 && p.dqk % 64 == 0) {
      dim3 pg(p.batch * p.heads * nch, p.dqk / 64);
      mlstm_prescale_channels_kernel<<<pg, 32 * kPcSeg, 0, st>>>(p, Qs, Ks, decay, rho_e, nadd, unsafe, kc, level);
    } else if (pair) {
      dim3 pg(p.batch * p.heads * nch, (DK + 255) / 256);
      mlstm_prescale_kernel<__nv_bfloat16, 2><<<pg, 128, 0, st>>>(p, Qs, Ks, decay, rho_e, nadd, unsafe, kc, level,
                                                                  fqg);
    } else {
      dim3 pg(p.batch * p.heads * nch, (DK + 127) / 128);
      mlstm_prescale_kernel<__nv_bfloat16, 1><<<pg, 128, 0, st>>>(p, Qs, Ks, decay, rho_e, nadd, unsafe, kc, level,
                                                                  fqg);
    }
    return check_launch("hxm_mlstm_chunkwise_fwd (prescale)");
  };
  const size_t smem = L::kBytes + 1024;
  auto kern = mlstm_stream_kernel<DK>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dv + kDV - 1) / kDV, p.heads, p.batch);
  auto stream = [&](int kc, int want) {
    CUtensorMap mq, mk, mv;
    const uint64_t dd[4] = {(uint64_t)DK, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
    const uint64_t sd[3] = {(uint64_t)DK * 2, (uint64_t)p.seqlen * DK * 2, (uint64_t)p.heads * p.seqlen * DK * 2};
    const uint64_t dvd[4] = {(uint64_t)p.dv, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
    const uint64_t sv[3] = {(uint64_t)p.tv * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
    hxm_status s;
    const uint64_t sq[3] = {(uint64_t)p.tq * 2, (uint64_t)p.sq[1] * 2, (uint64_t)p.sq[0] * 2};
    if ((s = raw_q ? make_map_bf16_4d(&mq, p.q, dd, sq, "mlstm q", kc)
                   : make_map_bf16_4d(&mq, Qs, dd, sd, "mlstm Qs", kc)) != HXM_OK)
      return s;
    if ((s = make_map_bf16_4d(&mk, Ks, dd, sd, "mlstm Ks", kc)) != HXM_OK) return s;
    if ((s = make_map_bf16_4d(&mv, p.v, dvd, sv, "mlstm v", kc)) != HXM_OK) return s;
    kern<<<grid, kStreamThreads, smem, st>>>(mq, mk, mv, p, decay, rho_e, nadd, unsafe, kc, want, fqg);
    return check_launch("hxm_mlstm_chunkwise_fwd (stream)");
  };
  // 128-step chunks for every pair in range; the pairs out of it are prescaled again in 64-step
  // chunks (halving each chunk's exponent range) and run with those; the pairs out of range even
  // then take the exact recurrent kernel.  Each launch's other CTAs return at once.
  hxm_status s;
  if ((s = prescale(kC, 0)) != HXM_OK) return s;
  if ((s = stream(kC, 0)) != HXM_OK) return s;
  if ((s = prescale(kC / 2, 1)) != HXM_OK) return s;
  if ((s = stream(kC / 2, 1)) != HXM_OK) return s;
  return launch_recurrent(p, st, unsafe, 2);
}

hxm_status launch_stream(const Params& p, cudaStream_t st) {
  if (p.dqk == 128) return launch_stream_dk<128>(p, st);
  if (p.dqk == 256) return launch_stream_dk<256>(p, st);
  return launch_stream_dk<512>(p, st);
}

}  // namespace mlstm
}  // namespace hxm
