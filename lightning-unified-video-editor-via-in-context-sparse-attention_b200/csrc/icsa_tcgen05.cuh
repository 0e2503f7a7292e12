// tcgen05 (5th-generation tensor core) helpers: tensor-memory allocation,
// shared-memory operand descriptors, MMA issue, commit, and TMEM<->register
// moves.  Inline PTX, single-CTA (cta_group::1) forms only.
#pragma once

#include "icsa_common.cuh"

namespace icsa {
namespace tc {

// ---- tensor memory allocation (one warp executes these) -------------------
ICSA_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
ICSA_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
ICSA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

ICSA_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ICSA_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- descriptors -----------------------------------------------------------
// Shared-memory matrix descriptor for a 128-byte-swizzled operand.
//   K-major operand: rows of 128 B (64 bf16 of K), 8-row atoms of 1024 B;
//                    SBO = 1024 (atom stride), LBO unused (1).
//   MN-major operand: rows of 128 B (64 bf16 of M/N) per K index, 8 K-rows per
//                    1024 B atom (SBO), next 64-wide M/N chunk at LBO.
ICSA_DEV uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  d |= uint64_t(2) << 61;  // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and an fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                      // D format: f32
         | (1u << 7)                    // A format: bf16
         | (1u << 10)                   // B format: bf16
         | (uint32_t(a_mn_major) << 15) // A major-ness
         | (uint32_t(b_mn_major) << 16) // B major-ness
         | (uint32_t(N >> 3) << 17)     // N / 8
         | (uint32_t(M >> 4) << 24);    // M / 16
}

// ---- MMA + commit ----------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T   (both described by descriptors)
ICSA_DEV void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T.  A (M=128 x K=16 bf16 per instruction)
// sits in 8 consecutive TMEM columns, lane = row, two bf16 per 32-bit column
// (element 2c in the low half of column c).
ICSA_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same as mma_bf16_ss / mma_bf16_ts with compile-time offsets added to the
// descriptors (and the A TMEM address) inside the instruction block, so the
// per-K-step operands are never materialised in registers.
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_bf16_ss_off(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ta, tb;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s64 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ta, tb, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}

template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_bf16_ts_off(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 ta;\n\t.reg .b64 tb;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s32 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], tb, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}

// Warp-converged forms: every lane of the issuing warp executes them and the
// lane chosen by elect.sync issues.  A converged issuing warp keeps the
// descriptor arithmetic warp-uniform, which issues much faster than a single
// diverged lane.
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_bf16_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 ta, tb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s64 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ta, tb, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_bf16_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 ta;\n\t.reg .b64 tb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s32 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], tb, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}
ICSA_DEV void mma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
ICSA_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- TMEM <-> registers (32 lanes x 32-bit, 32 consecutive columns) -------
#define ICSA_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define ICSA_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

ICSA_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : ICSA_R8(0), ICSA_R8(8), ICSA_R8(16), ICSA_R8(24)
      : "r"(taddr)
      : "memory");
}

ICSA_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      ICSA_W8(0), ICSA_W8(8), ICSA_W8(16), ICSA_W8(24)
      : "memory");
}

// 16 consecutive columns
ICSA_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : ICSA_R8(0), ICSA_R8(8)
      : "r"(taddr)
      : "memory");
}

ICSA_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      ICSA_W8(0), ICSA_W8(8)
      : "memory");
}

#undef ICSA_R8
#undef ICSA_W8

ICSA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
ICSA_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Per-warp register budget changes (all threads of the warp execute these).
template <uint32_t N>
ICSA_DEV void reg_alloc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <uint32_t N>
ICSA_DEV void reg_dealloc() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

}  // namespace tc
}  // namespace icsa
