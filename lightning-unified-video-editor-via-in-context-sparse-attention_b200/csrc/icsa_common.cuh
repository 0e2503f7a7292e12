// Shared definitions for the in-context sparse attention kernels (sm_100a).
//
// Everything here is plain CUDA C++ plus inline PTX for the Blackwell
// asynchronous machinery: mbarriers, TMA tensor loads (each CTA loads for itself),
// and the tcgen05 tensor-memory / MMA instructions.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "icsa.h"

#define ICSA_DEV __device__ __forceinline__

namespace icsa {

constexpr int kBlock = 64;          // BLOCK_M of the reference: tokens per block
constexpr int kTileRows = 128;      // Q rows per attention tile (two 64-token blocks)

// ---------------------------------------------------------------------------
// Chained launches (programmatic dependent launch).  A kernel launched with
// launch_chained may start while the kernel before it in the stream is still
// finishing; it calls wait_prior_grid() before it reads anything that kernel
// wrote (the wait returns once the prior grid has completed and its memory
// is visible).  Kernels launched without the attribute pass the wait at once.
// ---------------------------------------------------------------------------
ICSA_DEV void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... Params, typename... Args>
inline cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// ---------------------------------------------------------------------------
// Error reporting from device code.  Every bounded wait that gives up writes a
// code into the call's status word `err` (first writer wins) and the kernel
// winds down instead of hanging.
//
// The same code also goes into g_sticky_status, a per-device record that
// outlives the call's workspace: icsa_last_status() reads (and clears) it, so
// a caller that has discarded the workspace still learns that a wait gave up.
// The variable is file-scope static, so every translation unit that includes
// this header has its own copy; the units whose kernels wait define an
// accessor with ICSA_DEFINE_STICKY_ACCESSOR and icsa_capi.cu reads them all.
// ---------------------------------------------------------------------------
static __device__ int g_sticky_status;

ICSA_DEV void report_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
  atomicCAS(&g_sticky_status, 0, code);
}

// Host accessor of this translation unit's copy of g_sticky_status.
#define ICSA_DEFINE_STICKY_ACCESSOR(fn)                                    \
  cudaError_t fn(int** out) {                                              \
    return cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_sticky_status); \
  }

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
ICSA_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

ICSA_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Order-preserving map from float to uint32 (larger float -> larger uint).
// -0.0 is folded onto +0.0 first so that the two compare equal, as they do
// under IEEE comparison.
ICSA_DEV uint32_t float_order_key(float v) {
  v = v + 0.0f;
  uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit selection key: sorting keys in DESCENDING order yields values in
// descending order with ties broken towards the LOWER index.
ICSA_DEV uint64_t select_key(float v, uint32_t idx) {
  return (uint64_t(float_order_key(v)) << 32) | uint64_t(0xFFFFFFFFu - idx);
}
ICSA_DEV uint32_t select_key_index(uint64_t key) { return 0xFFFFFFFFu - uint32_t(key & 0xFFFFFFFFu); }

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
ICSA_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
ICSA_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

ICSA_DEV void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ICSA_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

ICSA_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

ICSA_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Non-blocking probe of a phase (never suspends the thread).
ICSA_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

ICSA_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete, giving up after about
// one second.  Returns false (and records `code` in *err) on timeout.  Once any
// wait in the kernel has failed (`*abort_flag` set), later waits return at
// once so that every role of the kernel reaches its exit path.
ICSA_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((it & 63u) == 63u) {
      uint64_t now = global_timer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > 1000000000ull) {
        report_error(err, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Same contract as mbar_wait, but polls with the non-suspending test: the
// caller wakes as soon as the phase completes.  For a single thread whose
// reaction time is on the critical path (the MMA issuer).
ICSA_DEV bool mbar_spin_wait(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_test_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((it & 1023u) == 1023u) {
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

// ---------------------------------------------------------------------------
// TMA (tensor) loads.  Single-CTA form only: each load lands in the issuing CTA.
// ---------------------------------------------------------------------------
ICSA_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

ICSA_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// TMA store of one box from this CTA's shared memory (bulk-group completion).
ICSA_DEV void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
ICSA_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store of this thread has completed.
ICSA_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Waits until every committed bulk store of this thread has read its shared
// memory source (the global writes complete asynchronously), which is what a
// CTA needs before it releases that shared memory.
ICSA_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

ICSA_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (tensor
// core reads of operands written with st.shared).
ICSA_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace icsa
