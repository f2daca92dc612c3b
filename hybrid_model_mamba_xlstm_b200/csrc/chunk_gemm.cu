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
// A CTA computes one 128 x BN tile of one group.  One elected thread issues the TMA
// loads (128-byte swizzle, 64-element K slices) into a 3-stage ring and the MMAs
// (M = 128, N = BN, K = 16 per instruction); the four warps then read the accumulator
// rows back (warp w: TMEM lanes 32w..32w+31, one row per thread) for the epilogue.
// Operands stored transposed relative to the product are read MN-major by the MMA
// (no transpose pass).  Rows / columns past a stored extent are zero-filled by TMA, so
// ragged M, N, K (a 64-step chunk in a 128-row tile, w = dv + 1 columns) need no
// padding copies; the epilogue stores only rows < M and columns < N.
//
// Every mbarrier wait is bounded (wait_limit cycles): on give-up the CTA raises the
// caller's error word, lets its own loads and MMAs land, frees its TMEM and returns.
#include "capi_internal.h"
#include "tc_sm100.cuh"
#include "tma_host.h"

namespace hxm {
namespace cgemm {

constexpr int kBM = 128;      // tile rows = TMEM lanes = MMA M
constexpr int kBK = 64;       // K slice per stage (one 128-byte swizzle row of bf16)
constexpr int kStages = 3;
constexpr int kThreads = 128;
constexpr int kPanel = 64 * 128;  // one MN-major panel: 64 K rows x 64 elements (8 KB)
constexpr long long kDrain = 200000000ll;
constexpr int kMaxProd = 4;

struct Params {
  int M, N, ksteps[kMaxProd];
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

template <int BN>
struct Smem {
  static constexpr int kA = kBM * 128;  // 128 rows x 128 B, or two MN panels
  static constexpr int kB = BN * 128;   // BN rows x 128 B, or BN / 64 MN panels
  static constexpr int kStage = kA + kB;
  static constexpr int kBar = kStages * kStage;
  static constexpr size_t kBytes = kBar + 8 * (2 * kStages + 1) + 16 + 1024;  // + 1024-byte alignment slack
};

// The TMA loads of one K slice: A as 128 rows of the slice (stored (M, K)) or two 64-wide
// M panels (stored (K, M)); B as BN rows (stored (N, K)) or BN / 64 panels (stored (K, N)).
template <int BN>
HXM_DEV void issue_loads(const CUtensorMap* ma, const CUtensorMap* mb, int a_mn, int b_mn, unsigned char* sa,
                         unsigned char* sb, uint64_t* bar, int m0, int n0, int k0, int g) {
  if (a_mn) {
    tc::tma_load_4d(sa, ma, bar, m0, k0, g, 0);
    tc::tma_load_4d(sa + kPanel, ma, bar, m0 + 64, k0, g, 0);
  } else {
    tc::tma_load_4d(sa, ma, bar, k0, m0, g, 0);
  }
  if (b_mn) {
#pragma unroll
    for (int q = 0; q < BN / 64; ++q) tc::tma_load_4d(sb + q * kPanel, mb, bar, n0 + 64 * q, k0, g, 0);
  } else {
    tc::tma_load_4d(sb, mb, bar, k0, n0, g, 0);
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads) chunk_gemm_kernel(
    const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap mb0,
    const __grid_constant__ CUtensorMap ma1, const __grid_constant__ CUtensorMap mb1,
    const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap mb2,
    const __grid_constant__ CUtensorMap ma3, const __grid_constant__ CUtensorMap mb3, const Params p) {
  using S = Smem<BN>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + S::kBar);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ int abort_flag, never;  // never: stays 0 (the drain waits ignore the abort)
  volatile int* abortp = &abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM, g = blockIdx.z;
  const uint32_t sbase = smem_u32(sm);

  if (tid == 0) {
    abort_flag = 0;
    never = 0;
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&ma0);
    tc::prefetch_tmap(&mb0);
  }
  if (warp == 0) tc::tmem_alloc(tmem_slot, BN);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool good = true;
  if (tid == 0) {
    // (the per-product fields are read as scalars: a runtime index into the by-value
    // parameter struct would copy it to local memory)
    const int e0 = p.ksteps[0], e1 = e0 + p.ksteps[1], e2 = e1 + p.ksteps[2], total = e2 + p.ksteps[3];
    const int amn0 = p.a_mn[0], amn1 = p.a_mn[1], amn2 = p.a_mn[2], amn3 = p.a_mn[3];
    const int bmn0 = p.b_mn[0], bmn1 = p.b_mn[1], bmn2 = p.b_mn[2], bmn3 = p.b_mn[3];
    // product of K slice j and the slice's index inside it
    auto prod_of = [&](int j) { return (j >= e0) + (j >= e1) + (j >= e2); };
    auto first_of = [&](int pi) { return pi == 0 ? 0 : (pi == 1 ? e0 : (pi == 2 ? e1 : e2)); };
    int loaded = 0, consumed = 0;
    bool ok = true;
    // iteration it: TMA for K slice it into stage it % kStages (after the MMAs of that stage's
    // previous use), then the MMAs of slice it - (kStages - 1)
    for (int it = 0; it < total + kStages - 1 && ok; ++it) {
      if (it < total) {
        const int s = it % kStages;
        if (it >= kStages && !tc::mbar_wait(&empty[s], ((it / kStages) - 1) & 1, abortp, p.wait_limit)) {
          ok = false;
          break;
        }
        const int pi = prod_of(it);
        const int k0 = (it - first_of(pi)) * kBK;
        unsigned char* sa = sm + s * S::kStage;
        tc::mbar_expect_tx(&full[s], S::kStage);
        // each map is named directly (a runtime choice of map pointer would copy a map to local memory)
        if (pi == 0) issue_loads<BN>(&ma0, &mb0, amn0, bmn0, sa, sa + S::kA, &full[s], m0, n0, k0, g);
        else if (pi == 1) issue_loads<BN>(&ma1, &mb1, amn1, bmn1, sa, sa + S::kA, &full[s], m0, n0, k0, g);
        else if (pi == 2) issue_loads<BN>(&ma2, &mb2, amn2, bmn2, sa, sa + S::kA, &full[s], m0, n0, k0, g);
        else issue_loads<BN>(&ma3, &mb3, amn3, bmn3, sa, sa + S::kA, &full[s], m0, n0, k0, g);
        ++loaded;
      }
      const int i = it - (kStages - 1);
      if (i < 0) continue;
      const int s = i % kStages;
      if (!tc::mbar_wait(&full[s], (i / kStages) & 1, abortp, p.wait_limit)) {
        ok = false;
        break;
      }
      ++consumed;
      tc::tc_fence_after();
      const int pi = prod_of(i);
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
        tc::mma_bf16(tmem, tc::desc_add(da, kk * astep), tc::desc_add(db, kk * bstep), id, i > 0 || kk > 0);
      tc::mma_commit(&empty[s]);
    }
    tc::mma_commit(done);  // arrives once every MMA issued above has completed
    if (!ok) {
      // let the loads still in flight land before the shared memory is released
      for (int j = consumed; j < loaded; ++j) tc::mbar_wait(&full[j % kStages], (j / kStages) & 1, &never, kDrain);
      abort_flag = 1;
      good = false;
    }
  }
  if (good && !tc::mbar_wait(done, 0, abortp, p.wait_limit)) good = false;
  good = __syncthreads_and(good) && abort_flag == 0;
  tc::tc_fence_after();

  if (good) {
    const int r = m0 + 32 * warp + lane;
    const bool rv = r < p.M;
    const float br = (p.decay && rv) ? p.decay[(int64_t)g * p.decay_gs + r] : 0.f;
    float* orow = p.out ? p.out + (int64_t)g * p.out_gs + (int64_t)r * p.out_rs : nullptr;
    __nv_bfloat16* brow = p.outb ? p.outb + (int64_t)g * p.ob_gs + (int64_t)r * p.ob_rs : nullptr;
    __nv_bfloat16* lrow = p.outb_lo ? p.outb_lo + (int64_t)g * p.ob_gs + (int64_t)r * p.ob_rs : nullptr;
    const bool vec_out = orow && (reinterpret_cast<uintptr_t>(p.out) % 16 == 0) && p.out_gs % 4 == 0 && p.out_rs % 4 == 0;
    const bool vec_b = brow && (reinterpret_cast<uintptr_t>(p.outb) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(p.outb_lo) % 16 == 0) && p.ob_gs % 8 == 0 && p.ob_rs % 8 == 0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (n0 + c0 >= p.N) break;  // warp-uniform
      float v[32];
      tc::tmem_ld32(tc::taddr(tmem, 32 * warp, c0), v);
      tc::tmem_wait_ld();
      const int cb = n0 + c0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = v[j] * p.alpha;
        if (p.mask) {
          const int c = cb + j;
          if (c > r) x = 0.f;
          else if (p.decay) x *= expf(br - __ldg(p.decay + (int64_t)g * p.decay_gs + c));
        }
        v[j] = x;
      }
      if (!rv) continue;
      const bool full_cols = cb + 32 <= p.N;
      if (p.accumulate) {  // D += the output's current value (then every store below writes the sum)
        if (full_cols && vec_out) {
          const float4* o4 = reinterpret_cast<const float4*>(orow + cb);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 o = o4[q];
            v[4 * q] += o.x; v[4 * q + 1] += o.y; v[4 * q + 2] += o.z; v[4 * q + 3] += o.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (cb + j < p.N) v[j] += orow[cb + j];
        }
      }
      if (orow) {
        if (full_cols && vec_out) {
          float4* o4 = reinterpret_cast<float4*>(orow + cb);
#pragma unroll
          for (int q = 0; q < 8; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (cb + j < p.N) orow[cb + j] = v[j];
        }
      }
      if (brow) {
        // bf16 high part, and with outb_lo the low part bf16(v - high): together ~16 mantissa bits
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          __nv_bfloat16* dst = half == 0 ? brow : lrow;
          if (!dst) continue;
          if (full_cols && vec_b) {
            uint4* b4 = reinterpret_cast<uint4*>(dst + cb);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float x0 = v[8 * q + 2 * e], x1 = v[8 * q + 2 * e + 1];
                if (half) {
                  x0 -= __bfloat162float(__float2bfloat16_rn(x0));
                  x1 -= __bfloat162float(__float2bfloat16_rn(x1));
                }
                __nv_bfloat162 h2 = __floats2bfloat162_rn(x0, x1);
                w[e] = *reinterpret_cast<uint32_t*>(&h2);
              }
              b4[q] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float x = half ? v[j] - __bfloat162float(__float2bfloat16_rn(v[j])) : v[j];
              if (cb + j < p.N) dst[cb + j] = __float2bfloat16_rn(x);
            }
          }
        }
      }
    }
  } else if (tid == 0) {
    tc::mbar_wait(done, 0, &never, kDrain);  // the MMAs finish before TMEM is freed
    if (p.error_flag) atomicExch(p.error_flag, 1);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, BN);
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

template <int BN>
static hxm_status launch(const hxm_chunk_gemm_args* a, cudaStream_t st) {
  Params p{};
  p.M = a->m;
  p.N = a->n;
  CUtensorMap ma[kMaxProd], mb[kMaxProd];
  for (int i = 0; i < kMaxProd; ++i) {
    const int pi = i < a->nprod ? i : 0;
    const hxm_gemm_operand& A = a->a[pi];
    const hxm_gemm_operand& B = a->b[pi];
    p.a_mn[i] = A.trans ? 1 : 0;
    // B is MN-major when stored (K, N) (not transposed)
    p.b_mn[i] = B.trans ? 0 : 1;
    p.ksteps[i] = i < a->nprod ? (Op{&A}.k_len(true) + kBK - 1) / kBK : 0;
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
  const size_t smem = Smem<BN>::kBytes;
  auto kern = chunk_gemm_kernel<BN>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((a->n + BN - 1) / BN, (a->m + kBM - 1) / kBM, (unsigned)a->groups);
  kern<<<grid, kThreads, smem, st>>>(ma[0], mb[0], ma[1], mb[1], ma[2], mb[2], ma[3], mb[3], p);
  return check_launch("hxm_chunk_gemm");
}

}  // namespace cgemm
}  // namespace hxm

using hxm::cgemm::Op;

extern "C" hxm_status hxm_chunk_gemm(const hxm_chunk_gemm_args* a, void* stream) {
  hxm::clear_error();
  HXM_REQUIRE(a && a->struct_size == sizeof(hxm_chunk_gemm_args), "hxm_chunk_gemm: bad args / struct_size");
  HXM_REQUIRE(a->groups >= 0 && a->groups <= 65535, "hxm_chunk_gemm: groups %lld out of range [0, 65535]",
              (long long)a->groups);
  HXM_REQUIRE(a->m >= 0 && a->n >= 0 && a->nprod >= 1 && a->nprod <= 4, "hxm_chunk_gemm: bad m / n / nprod");
  HXM_REQUIRE(a->out || a->out_bf16, "hxm_chunk_gemm: no output");
  HXM_REQUIRE(!a->accumulate || a->out, "hxm_chunk_gemm: accumulate needs the fp32 output");
  HXM_REQUIRE(!a->out_bf16_lo || a->out_bf16, "hxm_chunk_gemm: out_bf16_lo needs out_bf16");
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
  if (a->n <= 64) return hxm::cgemm::launch<64>(a, st);
  return hxm::cgemm::launch<128>(a, st);
}
