// chunk_gemm.cu — batched chunk GEMMs on the tensor cores (tcgen05, sm_100a) for the
// chunkwise backward passes of the mLSTM and SSD recurrences.
//
// Per group g (one (batch, head, chunk) of the backward), with bf16 operands and fp32
// accumulation in TMEM:
//     D = alpha * sum_{p < nprod} op(A_p) op(B_p)          (M x N, nprod <= 4)
// then an element-wise epilogue on the accumulator: the causal mask of a chunk's
// step-by-step matrix (D[r, c] = 0 for c > r), optionally weighted by the decay
// exp(b_r - b_c) of a per-step cumulative log gate b, accumulation into an existing fp32
// output, and an fp32 and / or bf16 store (optionally with the bf16 low part, so that a
// product's fp32 result becomes a split operand of the next products).  The sums of products share one
// accumulator, so e.g. dQ = dS K + dN X^T is one launch and one store, and so is a
// product of fp32 operands split into bf16 high and low parts
// (A_hi B_hi + A_hi B_lo + A_lo B_hi, about 16 mantissa bits).
//
// Persistent, warp-specialized: one CTA per SM walks the (n tile, m tile, group) tiles of
// the launch; a tile is 128 x BN, BN a multiple of 16 chosen per call so that the tiles
// cover n evenly (264 = 2 x 144, 520 = 3 x 176: no 8-column remainder tiles).
//   warp 4 (one lane): TMA producer, streaming the 64-element K slices (128-byte swizzle)
//                      of successive tiles through a 4-stage shared-memory ring;
//   warp 5 (one lane): MMA issuer (M = 128, N = BN, K = 16 per instruction) into two
//                      TMEM accumulators used alternately;
//   warps 0-3:         epilogue of the previous tile while the next one loads and
//                      multiplies: warp w reads TMEM lanes 32w..32w+31 (one row per
//                      thread) and passes each 32 x 32 block through shared memory so
//                      that the stores are row-contiguous (four 128-byte rows per warp
//                      instruction).
// Operands stored transposed relative to the product are read MN-major by the MMA
// (no transpose pass).  Rows / columns past a stored extent are zero-filled by TMA, so
// ragged M, N, K (a 64-step chunk in a 128-row tile, w = dv + 1 columns) need no
// padding copies; the epilogue stores only rows < M and columns < N.
//
// Every mbarrier wait is bounded (wait_limit cycles): on give-up the CTA raises the
// caller's error word, lets its own loads and MMAs land, frees its TMEM and returns.
#include <algorithm>

#include "capi_internal.h"
#include "tc_sm100.cuh"
#include "tma_host.h"

namespace hxm {
namespace cgemm {

constexpr int kBM = 128;          // tile rows = TMEM lanes = MMA M
constexpr int kBK = 64;           // K slice per stage (one 128-byte swizzle row of bf16)
constexpr int kEpiWarps = 8;      // two per TMEM lane quarter (alternate 32-column blocks)
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 32 * (kEpiWarps + 2);
constexpr int kPanel = 64 * 128;  // one MN-major panel: 64 K rows x 64 elements (8 KB)
constexpr long long kDrain = 200000000ll;
constexpr int kMaxProd = 4;
constexpr int kPitch = 36;        // floats per row of a warp's 32 x 32 epilogue block (144 B)

struct Params {
  int M, N, BN, ntn, ntm, ntiles;  // tiles: n tiles x m tiles x groups
  int ksteps[kMaxProd];
  int nprod;       // products of the launch
  int interleave;  // 1: all products have the same K; their slices alternate (see the loops)
  int a_mn[kMaxProd], b_mn[kMaxProd];
  float alpha;
  int mask;
  const float* decay;
  int64_t decay_gs;
  int accumulate;
  float* out;
  int64_t out_gs, out_rs;
  __nv_bfloat16* outb;
  __nv_bfloat16* outb_lo;  // low part, same strides as outb (needs outb)
  int64_t ob_gs, ob_rs;
  int* error_flag;
  long long wait_limit;
};

// BNMAX: the largest tile width of the instantiation (TMEM columns per accumulator, B stage).
template <int BNMAX>
struct Smem {
  static constexpr int kStages = BNMAX <= 128 ? 4 : 3;
  static constexpr int kA = kBM * 128;     // 128 rows x 128 B, or two MN panels
  static constexpr int kB = BNMAX * 128;   // up to BNMAX rows x 128 B, or BNMAX / 64 MN panels
  static constexpr int kStage = kA + kB;
  static constexpr int kEpi = kStages * kStage;                 // epilogue blocks, one per warp
  static constexpr int kBar = kEpi + kEpiWarps * 32 * kPitch * 4;
  static constexpr int kNumBars = 2 * kStages + 2 + 2 + 1;      // full, empty, acc full, acc empty, done
  static constexpr size_t kBytes = kBar + 8 * kNumBars + 16 + 1024;  // + 1024-byte alignment slack
  static_assert(kBytes <= 227 * 1024, "one CTA per SM");
};

// The TMA loads of one K slice: A as 128 rows of the slice (stored (M, K)) or two 64-wide
// M panels (stored (K, M)); B as BN rows (stored (N, K)) or ceil(BN / 64) panels (stored
// (K, N)).
HXM_DEV void issue_loads(const CUtensorMap* ma, const CUtensorMap* mb, int a_mn, int b_mn, int BN,
                         unsigned char* sa, unsigned char* sb, uint64_t* bar, int m0, int n0, int k0, int g) {
  if (a_mn) {
    tc::tma_load_4d(sa, ma, bar, m0, k0, g, 0);
    tc::tma_load_4d(sa + kPanel, ma, bar, m0 + 64, k0, g, 0);
  } else {
    tc::tma_load_4d(sa, ma, bar, k0, m0, g, 0);
  }
  if (b_mn) {
    const int panels = (BN + 63) / 64;
    for (int q = 0; q < panels; ++q) tc::tma_load_4d(sb + q * kPanel, mb, bar, n0 + 64 * q, k0, g, 0);
  } else {
    tc::tma_load_4d(sb, mb, bar, k0, n0, g, 0);
  }
}

HXM_DEV void tile_origin(const Params& p, int t, int& n0, int& m0, int& g) {
  n0 = (t % p.ntn) * p.BN;
  const int r = t / p.ntn;
  m0 = (r % p.ntm) * kBM;
  g = r / p.ntm;
}

// One staged 32 x 32 block (rows row0.., columns cb..; wbuf rows of kPitch floats) to the
// outputs: lanes 8i..8i+7 take row 4 it + i, four columns each (a 128-byte fp32 row
// segment per 8 lanes).  Accumulate, then the fp32 and bf16 high / low stores; columns
// past ncap and rows past M are left alone.  The output flags are template parameters so
// that the row loop carries no branches on them.
template <bool ACC, bool OUT, bool BF, bool LO>
HXM_DEV void store_block(const Params& p, const float* wbuf, int lane, int g, int row0, int cb, int ncap) {
  const int col = cb + (lane & 7) * 4;
  const int rmax = min(32, p.M - row0);
  float* ob = OUT ? p.out + (int64_t)g * p.out_gs + (int64_t)row0 * p.out_rs + col : nullptr;
  const int64_t bo = (int64_t)g * p.ob_gs + (int64_t)row0 * p.ob_rs + col;
  const bool full = col + 4 <= ncap;
#pragma unroll 2
  for (int itr = 0; itr < 8; ++itr) {
    const int rr = 4 * itr + (lane >> 3);
    if (rr >= rmax) break;
    float4 x = reinterpret_cast<const float4*>(wbuf + rr * kPitch)[lane & 7];
    float* o = OUT ? ob + (int64_t)rr * p.out_rs : nullptr;
    const int64_t b = bo + (int64_t)rr * p.ob_rs;
    if (full) {
      if (ACC) {
        const float4 y = *reinterpret_cast<const float4*>(o);
        x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
      }
      if (OUT) *reinterpret_cast<float4*>(o) = x;
      if (BF) {
        const __nv_bfloat162 h01 = __floats2bfloat162_rn(x.x, x.y), h23 = __floats2bfloat162_rn(x.z, x.w);
        *reinterpret_cast<uint2*>(p.outb + b) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
        if (LO) {  // low parts: bf16(x - high)
          const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
          const __nv_bfloat162 l01 = __floats2bfloat162_rn(x.x - f01.x, x.y - f01.y);
          const __nv_bfloat162 l23 = __floats2bfloat162_rn(x.z - f23.x, x.w - f23.y);
          *reinterpret_cast<uint2*>(p.outb_lo + b) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
        }
      }
    } else {  // the tile's last columns
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (col + e >= ncap) break;
        float y = xs[e];
        if (ACC) y += o[e];
        if (OUT) o[e] = y;
        if (BF) {
          const __nv_bfloat16 h = __float2bfloat16_rn(y);
          p.outb[b + e] = h;
          if (LO) p.outb_lo[b + e] = __float2bfloat16_rn(y - __bfloat162float(h));
        }
      }
    }
  }
}

template <int BNMAX>
__global__ void __launch_bounds__(kThreads, 1) chunk_gemm_kernel(
    const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap mb0,
    const __grid_constant__ CUtensorMap ma1, const __grid_constant__ CUtensorMap mb1,
    const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap mb2,
    const __grid_constant__ CUtensorMap ma3, const __grid_constant__ CUtensorMap mb3, const Params p) {
  using S = Smem<BNMAX>;
  constexpr int kStages = S::kStages;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + S::kBar);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;  // [2]: accumulator ready (MMA -> epilogue)
  uint64_t* acce = accf + 2;         // [2]: accumulator drained (epilogue -> MMA)
  uint64_t* done = acce + 2;         // every MMA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int abort_flag, never, consumed_sh;  // never: stays 0 (the drain waits ignore the abort)
  volatile int* abortp = &abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BN = p.BN;
  const uint32_t sbase = smem_u32(sm);

  if (tid == 0) {
    abort_flag = 0;
    never = 0;
    consumed_sh = 0;
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], kEpiWarps);
    }
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc(tmem_slot, 2 * BNMAX);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // (the per-product fields are read as scalars: a runtime index into the by-value
  // parameter struct would copy it to local memory)
  const int e0 = p.ksteps[0], e1 = e0 + p.ksteps[1], e2 = e1 + p.ksteps[2], kt = e2 + p.ksteps[3];
  const int amn0 = p.a_mn[0], amn1 = p.a_mn[1], amn2 = p.a_mn[2], amn3 = p.a_mn[3];
  const int bmn0 = p.b_mn[0], bmn1 = p.b_mn[1], bmn2 = p.b_mn[2], bmn3 = p.b_mn[3];
  // K slice j of a tile: product-major, or — when every product has the same K — slice-major
  // with the products alternating, so that an operand shared by two products (the high part of
  // a split operand meets both parts of the other) is re-read from L2 right after its first
  // load instead of after the whole K loop of the product between them
  const int np = p.nprod, il = p.interleave;
  auto prod_of = [&](int j) { return il ? j % np : (j >= e0) + (j >= e1) + (j >= e2); };
  auto kslice_of = [&](int j, int pi) {
    return il ? j / np : j - (pi == 0 ? 0 : (pi == 1 ? e0 : (pi == 2 ? e1 : e2)));
  };

  int issued = 0;  // producer: K slices whose loads were issued
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tc::prefetch_tmap(&ma0);
      tc::prefetch_tmap(&mb0);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
        int n0, m0, g;
        tile_origin(p, t, n0, m0, g);
        for (int j = 0; j < kt; ++j, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !tc::mbar_wait(&empty[s], ((it / kStages) - 1) & 1, abortp, p.wait_limit)) {
            ok = false;
            break;
          }
          const int pi = prod_of(j);
          const int k0 = kslice_of(j, pi) * kBK;
          unsigned char* sa = sm + s * S::kStage;
          const int bmn = pi == 0 ? bmn0 : pi == 1 ? bmn1 : pi == 2 ? bmn2 : bmn3;
          tc::mbar_expect_tx(&full[s], kBM * 128 + (bmn ? ((BN + 63) / 64) * kPanel : BN * 128));
          // each map is named directly (a runtime choice of map pointer would copy a map to local memory)
          if (pi == 0) issue_loads(&ma0, &mb0, amn0, bmn0, BN, sa, sa + S::kA, &full[s], m0, n0, k0, g);
          else if (pi == 1) issue_loads(&ma1, &mb1, amn1, bmn1, BN, sa, sa + S::kA, &full[s], m0, n0, k0, g);
          else if (pi == 2) issue_loads(&ma2, &mb2, amn2, bmn2, BN, sa, sa + S::kA, &full[s], m0, n0, k0, g);
          else issue_loads(&ma3, &mb3, amn3, bmn3, BN, sa, sa + S::kA, &full[s], m0, n0, k0, g);
          ++issued;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x, ++tl) {
        const int buf = tl & 1;
        if (tl >= 2 && !tc::mbar_wait(&acce[buf], ((tl >> 1) - 1) & 1, abortp, p.wait_limit)) break;
        tc::tc_fence_after();
        const uint32_t acc = tmem + buf * BNMAX;
        for (int j = 0; j < kt; ++j, ++it) {
          const int s = it % kStages;
          if (!tc::mbar_wait(&full[s], (it / kStages) & 1, abortp, p.wait_limit)) {
            ok = false;
            break;
          }
          *reinterpret_cast<volatile int*>(&consumed_sh) = it + 1;
          tc::tc_fence_after();
          const int pi = prod_of(j);
          const uint32_t sa = sbase + s * S::kStage, sb = sa + S::kA;
          const bool amn = (pi == 0 ? amn0 : pi == 1 ? amn1 : pi == 2 ? amn2 : amn3) != 0;
          const bool bmn = (pi == 0 ? bmn0 : pi == 1 ? bmn1 : pi == 2 ? bmn2 : bmn3) != 0;
          const uint64_t da = amn ? tc::sdesc_sw128(sa, kPanel, 1024) : tc::sdesc_sw128(sa, 16, 1024);
          const uint64_t db = bmn ? tc::sdesc_sw128(sb, kPanel, 1024) : tc::sdesc_sw128(sb, 16, 1024);
          const uint32_t id = tc::idesc_bf16(kBM, BN, amn, bmn);
          // K = 16 per MMA: 32 bytes along a K-major row, 16 rows (2 KB) down an MN-major panel
          const uint32_t astep = amn ? 2048u : 32u, bstep = bmn ? 2048u : 32u;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::mma_bf16(acc, tc::desc_add(da, kk * astep), tc::desc_add(db, kk * bstep), id, j > 0 || kk > 0);
          tc::mma_commit(&empty[s]);
        }
        if (!ok) break;
        tc::mma_commit(&accf[buf]);
      }
      tc::mma_commit(done);  // arrives once every MMA issued above has completed
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4).. and the column blocks c0 = 32 (w / 4) + 64 i,
    // through its own 32 x 32 staging block
    const int quarter = warp & 3, half = warp >> 2;
    float* wbuf = reinterpret_cast<float*>(sm + S::kEpi) + warp * 32 * kPitch;
    const int mode = (p.accumulate ? 1 : 0) | (p.out ? 2 : 0) | (p.outb ? 4 : 0) | (p.outb_lo ? 8 : 0);
    int tl = 0;
    for (int t = blockIdx.x; t < p.ntiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (!tc::mbar_wait(&accf[buf], (tl >> 1) & 1, abortp, p.wait_limit)) break;
      tc::tc_fence_after();
      int n0, m0, g;
      tile_origin(p, t, n0, m0, g);
      const int row0 = m0 + 32 * quarter;
      const int r = row0 + lane;
      const float br = (p.decay && r < p.M) ? p.decay[(int64_t)g * p.decay_gs + r] : 0.f;
      const int ncap = min(p.N, n0 + BN);  // this tile's columns (TMEM columns past BN are not its own)
#pragma unroll 1
      for (int c0 = 32 * half; c0 < BN; c0 += 64) {
        const int cb = n0 + c0;
        if (cb >= ncap) break;  // warp-uniform
        float v[32];
        tc::tmem_ld32(tc::taddr(tmem + buf * BNMAX, 32 * quarter, c0), v);
        tc::tmem_wait_ld();
        if (p.alpha != 1.f) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
        }
        if (p.mask) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c = cb + j;
            if (c > r) v[j] = 0.f;
            else if (p.decay) v[j] *= expf(br - __ldg(p.decay + (int64_t)g * p.decay_gs + c));
          }
        }
        float4* srow = reinterpret_cast<float4*>(wbuf + lane * kPitch);
#pragma unroll
        for (int q = 0; q < 8; ++q) srow[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        __syncwarp();
        if (row0 < p.M) {
          switch (mode) {
            case 2: store_block<false, true, false, false>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 3: store_block<true, true, false, false>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 4: store_block<false, false, true, false>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 12: store_block<false, false, true, true>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 6: store_block<false, true, true, false>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 14: store_block<false, true, true, true>(p, wbuf, lane, g, row0, cb, ncap); break;
            case 7: store_block<true, true, true, false>(p, wbuf, lane, g, row0, cb, ncap); break;
            default: store_block<true, true, true, true>(p, wbuf, lane, g, row0, cb, ncap); break;
          }
        }
        __syncwarp();  // the block is read before the next one overwrites it
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[buf]);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp && lane == 0) tc::mbar_wait(done, 0, &never, kDrain);  // MMAs finish before TMEM is freed
  if (abort_flag) {
    if (warp == kProducerWarp && lane == 0) {
      // the loads issued but not consumed land before the shared memory is released
      const int consumed = *reinterpret_cast<volatile int*>(&consumed_sh);
      for (int j = consumed; j < issued; ++j) tc::mbar_wait(&full[j % kStages], (j / kStages) & 1, &never, kDrain);
    }
    if (tid == 0 && p.error_flag) atomicExch(p.error_flag, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 2 * BNMAX);
  }
}

// Stored extent, K-length, M / N length of an operand.
struct Op {
  const hxm_gemm_operand* o;
  int k_len(bool is_a) const { return is_a ? (o->trans ? o->rows : o->cols) : (o->trans ? o->cols : o->rows); }
  int mn_len(bool is_a) const { return is_a ? (o->trans ? o->cols : o->rows) : (o->trans ? o->rows : o->cols); }
};

static hxm_status make_operand_map(CUtensorMap* map, const hxm_gemm_operand& o, int64_t groups, uint32_t box_rows,
                                   const char* who) {
  const uint64_t dims[4] = {(uint64_t)o.cols, (uint64_t)o.rows, (uint64_t)groups, 1};
  const uint64_t gs = (uint64_t)o.group_stride * 2;
  const uint64_t st[3] = {(uint64_t)o.row_stride * 2, gs, gs * (uint64_t)groups};
  return make_map_bf16_4d(map, o.ptr, dims, st, who, box_rows);
}

// Tile width: the fewest tiles of at most 256 columns, each a multiple of 16 wide.
inline int tile_width(int n) {
  const int tiles = (n + 255) / 256;
  return ((n + tiles - 1) / tiles + 15) / 16 * 16;
}

template <int BNMAX>
static hxm_status launch(const hxm_chunk_gemm_args* a, int BN, cudaStream_t st) {
  Params p{};
  p.M = a->m;
  p.N = a->n;
  p.BN = BN;
  p.ntn = (a->n + BN - 1) / BN;
  p.ntm = (a->m + kBM - 1) / kBM;
  const int64_t ntiles = (int64_t)p.ntn * p.ntm * a->groups;
  HXM_REQUIRE(ntiles < (int64_t)0x7fffffff, "hxm_chunk_gemm: too many tiles (%lld)", (long long)ntiles);
  p.ntiles = (int)ntiles;
  CUtensorMap ma[kMaxProd], mb[kMaxProd];
  for (int i = 0; i < kMaxProd; ++i) {
    const int pi = i < a->nprod ? i : 0;
    const hxm_gemm_operand& A = a->a[pi];
    const hxm_gemm_operand& B = a->b[pi];
    p.a_mn[i] = A.trans ? 1 : 0;
    // B is MN-major when stored (K, N) (not transposed)
    p.b_mn[i] = B.trans ? 0 : 1;
    p.ksteps[i] = i < a->nprod ? (Op{&A}.k_len(true) + kBK - 1) / kBK : 0;
  }
  p.nprod = a->nprod;
  p.interleave = 1;
  for (int i = 1; i < a->nprod; ++i)
    if (p.ksteps[i] != p.ksteps[0]) p.interleave = 0;
  for (int i = 0; i < kMaxProd; ++i) {
    const int pi = i < a->nprod ? i : 0;
    const hxm_gemm_operand& A = a->a[pi];
    const hxm_gemm_operand& B = a->b[pi];
    hxm_status s;
    if ((s = make_operand_map(&ma[i], A, a->groups, A.trans ? 64 : kBM, "hxm_chunk_gemm A")) != HXM_OK) return s;
    if ((s = make_operand_map(&mb[i], B, a->groups, B.trans ? BN : 64, "hxm_chunk_gemm B")) != HXM_OK) return s;
  }
  p.alpha = a->alpha;
  p.mask = a->mask;
  p.decay = a->decay;
  p.decay_gs = a->decay_stride;
  p.accumulate = a->accumulate;
  p.out = a->out;
  p.out_gs = a->out_group_stride;
  p.out_rs = a->out_row_stride;
  p.outb = static_cast<__nv_bfloat16*>(a->out_bf16);
  p.outb_lo = static_cast<__nv_bfloat16*>(a->out_bf16_lo);
  p.ob_gs = a->outb_group_stride;
  p.ob_rs = a->outb_row_stride;
  p.error_flag = a->error_flag;
  p.wait_limit = a->wait_limit_cycles != 0 ? (long long)a->wait_limit_cycles : 4000000000ll;
  const size_t smem = Smem<BNMAX>::kBytes;
  auto kern = chunk_gemm_kernel<BNMAX>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  static int num_sms[64] = {0};
  int dev = 0;
  HXM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 64 && num_sms[dev] == 0)
    HXM_CUDA_TRY(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
  const int sms = dev < 64 ? num_sms[dev] : 148;
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sms);  // persistent: one CTA per SM
  kern<<<grid, kThreads, smem, st>>>(ma[0], mb[0], ma[1], mb[1], ma[2], mb[2], ma[3], mb[3], p);
  return check_launch("hxm_chunk_gemm");
}

}  // namespace cgemm
}  // namespace hxm

using hxm::cgemm::Op;

extern "C" hxm_status hxm_chunk_gemm(const hxm_chunk_gemm_args* a, void* stream) {
  hxm::clear_error();
  HXM_REQUIRE(a && a->struct_size == sizeof(hxm_chunk_gemm_args), "hxm_chunk_gemm: bad args / struct_size");
  HXM_REQUIRE(a->groups >= 0 && a->groups <= (1 << 24), "hxm_chunk_gemm: groups %lld out of range [0, 2^24]",
              (long long)a->groups);
  HXM_REQUIRE(a->m >= 0 && a->n >= 0 && a->nprod >= 1 && a->nprod <= 4, "hxm_chunk_gemm: bad m / n / nprod");
  HXM_REQUIRE(a->out || a->out_bf16, "hxm_chunk_gemm: no output");
  HXM_REQUIRE(!a->accumulate || a->out, "hxm_chunk_gemm: accumulate needs the fp32 output");
  HXM_REQUIRE(!a->out_bf16_lo || a->out_bf16, "hxm_chunk_gemm: out_bf16_lo needs out_bf16");
  HXM_REQUIRE(!a->out || (reinterpret_cast<uintptr_t>(a->out) % 16 == 0 && a->out_group_stride % 4 == 0 &&
                          a->out_row_stride % 4 == 0),
              "hxm_chunk_gemm: the fp32 output needs a 16-byte aligned base and strides of multiples of 4");
  HXM_REQUIRE(!a->out_bf16 || (reinterpret_cast<uintptr_t>(a->out_bf16) % 8 == 0 &&
                               reinterpret_cast<uintptr_t>(a->out_bf16_lo) % 8 == 0 &&
                               a->outb_group_stride % 4 == 0 && a->outb_row_stride % 4 == 0),
              "hxm_chunk_gemm: the bf16 outputs need 8-byte aligned bases and strides of multiples of 4");
  HXM_REQUIRE(!a->decay || a->mask, "hxm_chunk_gemm: the decay weighting applies to the causal mask");
  if (a->groups == 0 || a->m == 0 || a->n == 0) return HXM_OK;
  for (int i = 0; i < a->nprod; ++i) {
    const hxm_gemm_operand* ops[2] = {&a->a[i], &a->b[i]};
    for (int w = 0; w < 2; ++w) {
      const hxm_gemm_operand& o = *ops[w];
      HXM_REQUIRE(o.ptr && o.rows > 0 && o.cols > 0, "hxm_chunk_gemm: operand %c%d empty", w ? 'B' : 'A', i);
      HXM_REQUIRE(o.row_stride >= o.cols && o.row_stride % 8 == 0 && o.group_stride % 8 == 0 &&
                      reinterpret_cast<uintptr_t>(o.ptr) % 16 == 0,
                  "hxm_chunk_gemm: operand %c%d needs a 16-byte aligned base and strides of multiples of 8 "
                  "elements (row stride >= columns)",
                  w ? 'B' : 'A', i);
    }
    const Op A{&a->a[i]}, B{&a->b[i]};
    HXM_REQUIRE(A.mn_len(true) == a->m, "hxm_chunk_gemm: A%d has %d rows for m = %d", i, A.mn_len(true), a->m);
    HXM_REQUIRE(B.mn_len(false) == a->n, "hxm_chunk_gemm: B%d has %d columns for n = %d", i, B.mn_len(false), a->n);
    HXM_REQUIRE(A.k_len(true) == B.k_len(false), "hxm_chunk_gemm: inner lengths %d / %d differ", A.k_len(true),
                B.k_len(false));
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int bn = hxm::cgemm::tile_width(a->n);
  if (bn <= 128) return hxm::cgemm::launch<128>(a, bn, st);
  return hxm::cgemm::launch<256>(a, bn, st);
}

// ----------------------------------------------------------------------------------------
// hxm_scale_split: gate-scaled bf16 high / low operands, 8 columns per thread (16-byte
// output stores when cols % 8 == 0), one pass.
namespace hxm {
namespace cgemm {

template <typename T>
__global__ void __launch_bounds__(256) scale_split_kernel(const T* __restrict__ x, int64_t sb, int64_t st,
                                                          const float* __restrict__ scale, __nv_bfloat16* __restrict__ hi,
                                                          __nv_bfloat16* __restrict__ lo, int batch, int seqlen,
                                                          int lp, int cols, int group) {
  const int c8 = (cols + 7) / 8;
  const int64_t e = blockIdx.x * 256ll + threadIdx.x;
  if (e >= (int64_t)batch * lp * c8) return;
  const int cb = (int)(e % c8) * 8;
  const int64_t row = e / c8;
  const int t = (int)(row % lp), b = (int)(row / lp);
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = cb + j;
    float x0 = 0.f;
    if (t < seqlen && c < cols) {
      x0 = to_f32<T>(x[b * sb + (int64_t)t * st + c]);
      if (scale) x0 *= scale[row * (cols / group) + c / group];
    }
    v[j] = x0;
  }
  __nv_bfloat16 h[8], l[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    h[j] = __float2bfloat16_rn(v[j]);
    l[j] = __float2bfloat16_rn(v[j] - __bfloat162float(h[j]));
  }
  const int64_t o = row * cols + cb;
  if (cols % 8 == 0) {
    *reinterpret_cast<uint4*>(hi + o) = *reinterpret_cast<const uint4*>(h);
    if (lo) *reinterpret_cast<uint4*>(lo + o) = *reinterpret_cast<const uint4*>(l);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (cb + j < cols) {
        hi[o + j] = h[j];
        if (lo) lo[o + j] = l[j];
      }
  }
}

}  // namespace cgemm
}  // namespace hxm

extern "C" hxm_status hxm_scale_split(const hxm_scale_split_args* a, void* stream) {
  hxm::clear_error();
  HXM_REQUIRE(a && a->struct_size == sizeof(hxm_scale_split_args), "hxm_scale_split: bad args / struct_size");
  HXM_REQUIRE(a->batch >= 0 && a->seqlen >= 0 && a->padded_len >= a->seqlen && a->cols >= 1 && a->group >= 1 &&
                  a->cols % a->group == 0,
              "hxm_scale_split: bad sizes batch=%d seqlen=%d padded_len=%d cols=%d group=%d", a->batch, a->seqlen,
              a->padded_len, a->cols, a->group);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "hxm_scale_split: io_dtype must be f32 or bf16");
  const int64_t n = (int64_t)a->batch * a->padded_len * ((a->cols + 7) / 8);
  if (n == 0) return HXM_OK;
  HXM_REQUIRE(a->x && a->hi, "hxm_scale_split: NULL x or hi");
  HXM_REQUIRE(a->cols % 8 != 0 || (reinterpret_cast<uintptr_t>(a->hi) % 16 == 0 &&
                                    reinterpret_cast<uintptr_t>(a->lo) % 16 == 0),
              "hxm_scale_split: hi / lo need 16-byte alignment");
  const unsigned grid = (unsigned)((n + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* hi = static_cast<__nv_bfloat16*>(a->hi);
  auto* lo = static_cast<__nv_bfloat16*>(a->lo);
  if (a->io_dtype == HXM_F32)
    hxm::cgemm::scale_split_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(a->x), a->x_stride[0],
                                                                a->x_stride[1], a->scale, hi, lo, a->batch, a->seqlen,
                                                                a->padded_len, a->cols, a->group);
  else
    hxm::cgemm::scale_split_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(a->x), a->x_stride[0], a->x_stride[1], a->scale, hi, lo, a->batch,
        a->seqlen, a->padded_len, a->cols, a->group);
  return hxm::check_launch("hxm_scale_split");
}
