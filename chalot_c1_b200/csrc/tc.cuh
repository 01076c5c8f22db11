// tc.cuh — sm_100a tensor-core (tcgen05) and 2-D TMA helpers in inline PTX.
//
// Only what the int8 expert GEMM needs: TMEM allocation, the kind::i8 MMA
// with both operands K-major in 128-byte-swizzled shared memory, commits to
// mbarriers, TMEM loads of the 32x32b shape, and tiled 2-D TMA loads (no
// copy to other CTAs; every load reads this GPU's own memory).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "tma.cuh"

namespace chalot {

CHALOT_DEV void mbar_init_n(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CHALOT_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CHALOT_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tiled 2-D TMA load of box (c0 = innermost coordinate, c1) into `dst`,
// completing on `bar`. c0 * element size must be a multiple of 16 bytes.
CHALOT_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

CHALOT_DEV void tc_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
CHALOT_DEV void tc_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
CHALOT_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CHALOT_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (=|+=) A[smem] * B[smem]^T, signed int8 in, int32 out.
CHALOT_DEV void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar` when every MMA this thread issued before has completed.
CHALOT_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor of kind::i8: D s32, A and B s8, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_i8(int M, int N) {
  return (2u << 4)                    // D format: s32
         | (1u << 7) | (1u << 10)     // A, B format: signed 8-bit
         | ((uint32_t)(N >> 3) << 17)  // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor of a K-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart. The tile
// base is 1024-byte aligned; `saddr` may be advanced by k*32 bytes within the
// row to address the k-th 32-column slice.
CHALOT_DEV uint64_t tc_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                             // leading offset (unused when swizzled)
  d |= (uint64_t)(1024 >> 4) << 32;                   // stride offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                             // descriptor version
  d |= (uint64_t)2 << 61;                             // 128-byte swizzle
  return d;
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
CHALOT_DEV void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane.
CHALOT_DEV void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
CHALOT_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Writes the value v to 16 consecutive 32-bit TMEM columns of this thread's lane.
CHALOT_DEV void tc_st16_fill(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}

// Writes the value v to 32 consecutive 32-bit TMEM columns of this thread's lane.
CHALOT_DEV void tc_st32_fill(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
CHALOT_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed pairs of f32 (sm_100a f32x2 arithmetic, each lane rounded to nearest
// as the scalar .rn instruction rounds).
typedef unsigned long long f32x2;
CHALOT_DEV f32x2 f2_pack(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
CHALOT_DEV f32x2 f2_pack_bits(uint32_t lo, uint32_t hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
CHALOT_DEV void f2_unpack(f32x2 v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
CHALOT_DEV f32x2 f2_add(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
CHALOT_DEV f32x2 f2_sub(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
CHALOT_DEV f32x2 f2_mul(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
CHALOT_DEV f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// acc + p lane-wise with scalar add.rn.f32. A packed add (or fma(p, 1, acc))
// fed by a packed multiply was contracted into one fused multiply-add by the
// assembler despite .rn (measured: results then equal fma(x, y, acc)), also
// with the assembler's own contraction switched off (-Xptxas -fmad=false:
// the 4096-token layer then differs from the oracle); a scalar add with an
// explicit rounding modifier is never contracted.
CHALOT_DEV f32x2 f2_add_nc(f32x2 acc, f32x2 p) {
  float a0, a1, p0, p1;
  f2_unpack(acc, a0, a1);
  f2_unpack(p, p0, p1);
  return f2_pack(__fadd_rn(a0, p0), __fadd_rn(a1, p1));
}

}  // namespace chalot
