// tc_sm100.cuh — thin inline-PTX layer over the Blackwell (sm_100a) async
// machinery used by the chunkwise kernels: mbarriers with bounded waits, TMA
// tensor loads into this CTA only, TMEM allocation, tcgen05.mma / commit / ld / st,
// and the UMMA shared-memory + instruction descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 matrix descriptors" /
// "instruction descriptor" tables (the same fields CUTLASS names in
// cute/arch/mma_sm100_desc.hpp):
//   smem desc: [0,14) addr>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version=1,
//              [49,52) base offset, [52] LBO mode, [61,64) layout (2 = 128B swizzle)
//   idesc (kind::f16): [4,6) D fmt (1=f32), [7,10) A fmt (1=bf16), [10,13) B fmt,
//              [15] A MN-major, [16] B MN-major, [17,23) N>>3, [24,29) M>>4
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

#include "common.cuh"

namespace hxm {
namespace tc {

// ---------------------------------------------------------------- mbarrier --
HXM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
HXM_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
HXM_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
HXM_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
HXM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~`limit_cycles` SM cycles (or as soon as
// another thread of the CTA raised *abort), raising *abort.  Returns false
// on give-up.  Every wait of the kernels goes through this.
// The abort flag and the clock are checked every 32 polls only: a flag read
// per poll by every waiting thread competes with the tensor core for
// shared-memory bandwidth.
HXM_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, long long limit_cycles = 4000000000ll) {
  // a negative limit (the callers' error-path test) gives up before polling, whatever the barrier's state
  if (limit_cycles < 0) {
    *abort = 1;
    return false;
  }
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0) {
      if (*abort) return false;
      if (clock64() - t0 > limit_cycles) {
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------- fences --
HXM_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
HXM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
HXM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------------- TMA --
// Tiled 4-D load of a box into this CTA's shared memory, completing on `bar`.
HXM_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
HXM_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// --------------------------------------------------------------------- TMEM --
// Warp-wide: allocate `ncols` (power of two >= 32) columns, address written to *dst.
HXM_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HXM_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// TMEM address of (lane, column) relative to an allocation base.
HXM_DEV uint32_t taddr(uint32_t base, int lane, int col) { return base + ((uint32_t)lane << 16) + (uint32_t)col; }

// 32 consecutive fp32 columns of this thread's lane (warp w reads lanes 32*(w%4)..).
HXM_DEV void tmem_ld32(uint32_t addr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
}
HXM_DEV void tmem_st32(uint32_t addr, const float (&v)[32]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 16 consecutive fp32 columns of this thread's lane.
HXM_DEV void tmem_ld16(uint32_t addr, float (&v)[16]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
}
HXM_DEV void tmem_st16(uint32_t addr, const float (&v)[16]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// One fp32 column of this thread's lane.
HXM_DEV float tmem_ld1(uint32_t addr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(addr));
  return __uint_as_float(r);
}
HXM_DEV void tmem_st1(uint32_t addr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(addr), "r"(__float_as_uint(v)) : "memory");
}
HXM_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
HXM_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05 --
// D[tmem] (+)= A[smem] * B[smem]^T per the descriptors (one elected thread issues).
HXM_DEV void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// The same with compile-time byte offsets added to the two descriptors inside
// the instruction's own asm block: only the base descriptors stay live, and no
// per-MMA address arithmetic is scheduled ahead of the MMAs.
template <uint32_t AOFF, uint32_t BOFF>
HXM_DEV void mma_bf16_at(uint32_t d_tmem, uint64_t abase, uint64_t bbase, uint32_t idesc, bool accumulate) {
  static_assert(AOFF % 16 == 0 && BOFF % 16 == 0, "descriptor offsets are in 16-byte units");
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 a, b;\n\t"
      "add.s64 a, %1, %5;\n\t"
      "add.s64 b, %2, %6;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(abase), "l"(bbase), "r"(idesc), "r"((uint32_t)accumulate), "n"(AOFF >> 4), "n"(BOFF >> 4)
      : "memory");
}

// f(std::integral_constant<int, i>) for i = 0 .. N-1, unrolled at compile time.
template <typename F, int... I>
HXM_DEV void static_for_impl(F& f, std::integer_sequence<int, I...>) {
  (f(std::integral_constant<int, I>{}), ...);
}
template <int N, typename F>
HXM_DEV void static_for(F&& f) {
  static_for_impl(f, std::make_integer_sequence<int, N>{});
}

// Arrive on `bar` once every previously issued tcgen05 op of this thread completed.
HXM_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 128-byte-swizzled UMMA shared-memory descriptor.
//   K-major operand: rows of 64 bf16 (128 B), SBO = 1024 (8-row atoms), LBO unused (16).
//   MN-major operand: rows = K index holding 64 MN-contiguous bf16, SBO = 1024
//   (next 8 K rows), LBO = byte distance between 64-wide MN panels.
HXM_DEV uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// The descriptor of the same operand `bytes` further on (a multiple of 16):
// the start address field is the low 14 bits, and shared-memory addresses stay
// below 2^18, so the add never carries out of the field.  With a compile-time
// offset this is one integer add, which keeps the issuing thread's per-MMA
// instruction chain short (the issue loop, not the tensor core, otherwise
// sets the MMA rate).
HXM_DEV uint64_t desc_add(uint64_t desc, uint32_t bytes) { return desc + (uint64_t)(bytes >> 4); }

// kind::f16 instruction descriptor: bf16 x bf16 -> fp32, M x N tile.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (row, col) inside a 128B-swizzled panel of 64-element
// bf16 rows (the layout TMA SWIZZLE_128B writes and UMMA SW128 reads):
// 16-byte chunk (col/8) of row r sits at chunk position (col/8) ^ (r % 8).
HXM_DEV uint32_t sw128_offset(int row, int col) {
  return (uint32_t)row * 128u + ((((uint32_t)col >> 3) ^ ((uint32_t)row & 7u)) << 4) + (((uint32_t)col & 7u) << 1);
}

}  // namespace tc
}  // namespace hxm
