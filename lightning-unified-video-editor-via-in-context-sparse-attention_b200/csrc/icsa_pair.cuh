// Helpers for kernels that run on an SM pair (a cluster of two CTAs) and
// drive the tensor cores of both SMs with one instruction stream
// (tcgen05 cta_group::2).  Inline PTX.
//
// Division of labour in such a pair:
//   * both CTAs allocate the same TMEM columns (tcgen05.alloc.cta_group::2);
//   * the even CTA (cluster rank 0, the "leader") issues every tcgen05.mma.
//     A (M = 256) is split by rows: rows [0,128) come from the leader's shared
//     memory / TMEM, rows [128,256) from the peer's, at the same addresses.
//     B (N columns) is split by columns: the leader holds [0, N/2), the peer
//     [N/2, N).  Each CTA's TMEM receives its own 128 rows of D;
//   * each CTA loads its own operand halves with TMA and signals the leader's
//     "full" barrier, whose expected byte count covers both halves;
//   * the leader's commits arrive on the barrier at the same offset in both
//     CTAs (CTA mask 0b11), so each CTA waits on its own copy.
#pragma once

#include "icsa_tcgen05.cuh"

namespace icsa {
namespace pair {

ICSA_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs: barrier over the cluster with release/acquire
// ordering of shared-memory accesses.
ICSA_DEV void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Address in the cluster shared window of the variable that lives at `p` in
// this CTA, as seen in CTA `rank` of the cluster.
ICSA_DEV uint32_t mapa(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

// Arrive (count 1) on an mbarrier given by its cluster address (any CTA of
// the cluster, this one included).
ICSA_DEV void arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// Same with relaxed ordering: for arrivals whose only purpose is to report
// that this thread's tcgen05 loads or stores have completed (tcgen05.wait::ld /
// wait::st already returned), so no memory fence is needed before them.
ICSA_DEV void arrive_cluster_relaxed(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

ICSA_DEV bool try_wait(uint64_t* bar, uint32_t parity) {
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

ICSA_DEV bool test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded single-thread wait (about one second), cluster-scope acquire.
// Spinning with test_wait keeps the reaction time short for the MMA issuer.
ICSA_DEV bool wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag, bool spin = false) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (spin ? test_wait(bar, parity) : try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((it & 255u) == 255u) {
      const uint64_t now = global_timer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > 1000000000ull) {
        report_error(err, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Warp-uniform bounded wait (all lanes poll; the warp gives up together).
ICSA_DEV bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag) {
  bool done = try_wait(bar, parity);
  uint64_t t0 = 0;
  uint32_t it = 0;
  while (!__all_sync(0xffffffffu, done)) {
    if (!done) done = try_wait(bar, parity);
    bool give_up = *abort_flag != 0;
    if ((threadIdx.x & 31) == 0 && (++it & 63u) == 0u) {
      const uint64_t now = global_timer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > 1000000000ull) {
        report_error(err, code);
        *abort_flag = 1;
        give_up = true;
      }
    }
    if (__any_sync(0xffffffffu, give_up)) return false;
  }
  return true;
}

// ---- tensor memory for the pair (one warp of EACH CTA, same warp index) ----
ICSA_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
ICSA_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
ICSA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- MMA over the pair (issued by one thread of the leader) ---------------
// D[tmem] (+)= A[smem] * B[smem]^T with compile-time descriptor offsets.
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ta, tb;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s64 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], ta, tb, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T.
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 ta;\n\t.reg .b64 tb;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s32 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [ta], tb, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}

// Warp-converged forms: every lane of the issuing warp executes them and one
// lane, chosen by elect.sync, issues the instruction.  Keeping the issuing
// warp converged lets the descriptors stay warp-uniform.
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 ta, tb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s64 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], ta, tb, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}
template <uint32_t AOFF, uint32_t BOFF>
ICSA_DEV void mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 ta;\n\t.reg .b64 tb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "add.s32 ta, %1, %5;\n\t"
      "add.s64 tb, %2, %6;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [ta], tb, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(AOFF), "n"(BOFF)
      : "memory");
}
ICSA_DEV void commit_both_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "mov.b16 m, 3;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Arrive once on the mbarrier at this offset in both CTAs of the pair when
// all previously issued pair MMAs of this thread have completed.
ICSA_DEV void commit_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---- TMA load into this CTA's shared memory, completing bytes on the
// leader's barrier (given by its cluster address). ---------------------------
ICSA_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int c0, int c1, int c2,
                          int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 2-D form of tma_load_4d.
ICSA_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

// Named barrier over `count` threads (whole warps).
ICSA_DEV void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Arrive on a named barrier without waiting (the producer side of a
// producer/consumer hand-off; the consumer uses named_sync).
ICSA_DEV void named_arrive(uint32_t id, uint32_t count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace pair
}  // namespace icsa
