// Deterministic in-shared-memory sorting used by every block selection.
#pragma once

#include "icsa_common.cuh"

namespace icsa {

// ---------------------------------------------------------------------------
// Bitonic sort, descending, over a shared-memory array of pow2 length (>= 32)
// by the `nthreads` threads of a CTA (a multiple of 32; thread t handles
// elements t, t + nthreads, ...).  A compare-exchange stage of stride j < 32
// pairs elements of one 32-aligned segment, and every element of a segment
// is handled by one warp, so between two such stages a warp barrier
// suffices; a CTA barrier follows every stage that has, or is followed by a
// stage that has, a stride of 32 or more.
// ---------------------------------------------------------------------------
template <typename T>
ICSA_DEV void bitonic_sort_desc(T* a, int n, int tid, int nthreads) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n; i += nthreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          T x = a[i], y = a[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      const int next_j = j > 1 ? j >> 1 : k;  // first stride of the next k
      if (j >= 32 || next_j >= 32 || k == n) __syncthreads();
      else __syncwarp();
    }
  }
}

inline int next_pow2(int n) {
  int p = 32;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace icsa

namespace icsa {

// ---------------------------------------------------------------------------
// Warp-level radix select.  `keys` (shared memory, n entries) hold
// order-preserving 32-bit keys (float_order_key).  Returns the key of the
// k-th largest entry (1 <= k <= n) and sets *n_greater to the number of
// entries strictly greater than it.  Four passes over 8-bit digits with a
// 256-bin shared-memory histogram `hist` private to the warp.  Every lane
// returns the same values.
// ---------------------------------------------------------------------------
ICSA_DEV uint32_t warp_kth_largest(const uint32_t* keys, int n, int k, uint32_t* hist, int* n_greater) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0;  // digits fixed so far (high bits)
  int remaining = k;    // rank still to find inside the current prefix bucket
  int greater = 0;      // entries above the current prefix bucket
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int i = lane; i < n; i += 32) {
      const uint32_t u = keys[i];
      if ((u & hi_mask) == (prefix & hi_mask)) atomicAdd(&hist[(u >> shift) & 255u], 1u);
    }
    __syncwarp();
    // lane L owns bins 255-8L .. 248-8L (descending); find the bin where the
    // cumulative count from the top reaches `remaining`.
    uint32_t c[8];
    uint32_t local = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      c[e] = hist[255 - 8 * lane - e];
      local += c[e];
    }
    uint32_t incl = local;  // inclusive scan over lanes (from the top bins down)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const uint32_t excl = incl - local;
    const bool mine = excl < uint32_t(remaining) && incl >= uint32_t(remaining);
    uint32_t digit = 0, above = 0;
    if (mine) {
      uint32_t run = excl;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (run + c[e] >= uint32_t(remaining)) {
          digit = 255 - 8 * lane - e;
          above = run;
          break;
        }
        run += c[e];
      }
    }
    const unsigned owner = __ballot_sync(0xffffffffu, mine);
    const int src = __ffs(owner) - 1;
    digit = __shfl_sync(0xffffffffu, digit, src);
    above = __shfl_sync(0xffffffffu, above, src);
    prefix |= digit << shift;
    greater += int(above);
    remaining -= int(above);
    __syncwarp();
  }
  *n_greater = greater;
  return prefix;
}

}  // namespace icsa
