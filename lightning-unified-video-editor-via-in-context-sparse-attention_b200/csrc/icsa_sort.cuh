// Deterministic in-shared-memory sorting used by every block selection.
#pragma once

#include "icsa_common.cuh"

namespace icsa {

// ---------------------------------------------------------------------------
// Bitonic sort, descending, over a shared-memory array of pow2 length, by a
// group of `nthreads` threads (a warp or the whole CTA); `sync` is the
// matching barrier.
// ---------------------------------------------------------------------------
template <typename T, typename Sync>
ICSA_DEV void bitonic_sort_desc(T* a, int n, int tid, int nthreads, Sync sync) {
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
      sync();
    }
  }
}

struct WarpSync {
  ICSA_DEV void operator()() const { __syncwarp(); }
};
struct BlockSync {
  ICSA_DEV void operator()() const { __syncthreads(); }
};

inline int next_pow2(int n) {
  int p = 32;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace icsa
