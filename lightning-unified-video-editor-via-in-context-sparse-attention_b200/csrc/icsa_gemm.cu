// Linear layer with the residual update fused into its epilogue, on SM pairs
// (tcgen05 cta_group::2), for the DiT block's output projections:
//
//   x[r, c] += bf16( a[r, :] . w[c, :] + bias[c] ) * gate[r / rows_per_batch, c]
//
// (gate NULL: x[r, c] += bf16(...)).  This is the reference's
// `x = x + self.o(y) * e[2]` (model.py:175-176 with :258-259), the
// cross-attention's `x = x + self.cross_attn(...)` (:262, o-projection
// :188) and the FFN's `x = x + y * e[5]` (:263-265), where the nn.Linear runs
// in bf16 under autocast: float32 accumulation plus bias, rounded once to
// bf16, then the product and the sum in float32, each rounded once.  The
// bf16 y and the separate residual pass over the float32 stream disappear.
//
// Tiles: a cluster of two CTAs computes a 256 x 256 tile of the output, each
// CTA 128 rows; per K step of 128 each CTA loads its 128 x 128 slice of a and
// its 128 x 128 half of the 256 weight rows with TMA (two 64-wide atoms of
// 16 KB each, 128-byte swizzle), and the leader issues eight M = 256,
// N = 256, K = 16 MMAs for the pair.  Per SM that is 64 KB of shared memory
// read by the tensor core and 64 KB written by TMA per 1024 clk of tensor
// work; one wait and one commit per 1024 clk keep the MMA warp's own
// overheads off the tensor core's path.
//
// The kernel is persistent: every cluster walks the tile list with a stride
// of the cluster count, in groups of kGGroupM tile rows (tile rows fastest
// within a group), so the clusters running at one time share their rows of
// a and their columns of w in L2.  TMEM holds two 256-column accumulators:
// the epilogue of one tile runs while the MMAs of the next one fill the
// other.
//
// Roles per CTA (192 threads): warps 0-3 epilogue (thread <-> TMEM lane <->
// output row), warp 4 TMA producer, warp 5 TMEM allocation and, in the
// leader, the MMA issuer.  Every wait is bounded (about one second); a wait
// that gives up records a status code (report_error) and the kernel winds
// down.
#include "icsa_attn_common.cuh"
#include "icsa_pair.cuh"

#include <algorithm>

#include <utility>

namespace icsa {

namespace {

constexpr int kGThreads = 192;
constexpr int kGProducerWarp = 4;
constexpr int kGMmaWarp = 5;
#ifndef ICSA_GEMM_ATOMS
#define ICSA_GEMM_ATOMS 2
#endif
#ifndef ICSA_GEMM_GROUP_M
#define ICSA_GEMM_GROUP_M 8
#endif
constexpr int kGAtoms = ICSA_GEMM_ATOMS;             // 64-wide K atoms (128-byte swizzled rows) per stage
constexpr int kGStages = 6 / kGAtoms;
constexpr int kGRows = 128;                          // output rows per CTA (256 per pair)
constexpr int kGCols = 256;                          // output columns per pair tile
constexpr int kGAtomK = 64;                          // K of one atom
constexpr int kGKStep = kGAtomK * kGAtoms;           // K per stage
constexpr int kGAtomBytes = 128 * kGAtomK * 2;       // 16 KB: 128 rows of one atom
constexpr int kGABytes = kGAtoms * kGAtomBytes;      // this CTA's 128 rows of a
constexpr int kGBBytes = kGAtoms * kGAtomBytes;      // this CTA's 128 of the 256 weight rows
constexpr uint32_t kGTmemCols = 512;                 // two accumulators of 256 columns
constexpr int kGGroupM = ICSA_GEMM_GROUP_M;          // tile rows per raster group

enum : int { kErrGFull = 0x301, kErrGEmpty = 0x302, kErrGAccFull = 0x303, kErrGAccEmpty = 0x304, kErrGDrain = 0x305 };

struct GemmParams {
  int M, N, K;
  const __nv_bfloat16* bias;  // [N] or nullptr
  float* x;                   // [M, ldx] float32 residual stream
  int64_t ldx;
  const float* gate;          // row b at b * gate_bs, or nullptr
  int64_t gate_bs;
  int rows_per_batch;
  int m_tiles, n_tiles, tiles, k_steps;
};

struct GemmMaps {
  CUtensorMap a;  // bf16 [M, K], box {64, 128}
  CUtensorMap w;  // bf16 [N, K], box {64, 128}
};

struct __align__(1024) GSmem {
  uint8_t a[kGStages][kGABytes];
  uint8_t b[kGStages][kGBBytes];
  uint64_t full[kGStages], empty[kGStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(GSmem) + 1024 <= 232448, "gemm kernel shared memory exceeds 227 KB");

ICSA_DEV void tile_coords(const GemmParams& p, int t, int& mt, int& nt) {
  const int group = kGGroupM * p.n_tiles;
  const int g = t / group, r = t - g * group;
  const int m0 = g * kGGroupM;
  const int gm = min(kGGroupM, p.m_tiles - m0);
  mt = m0 + r % gm;
  nt = r / gm;
}

ICSA_DEV void gemm_producer(const GemmParams& p, const GemmMaps& maps, GSmem& sm, uint32_t rank, int* issued) {
  volatile int* abort_flag = &sm.abort_flag;
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  int it = 0;
  for (int t = cluster; t < p.tiles; t += clusters) {
    int mt, nt;
    tile_coords(p, t, mt, nt);
    const int row0 = mt * (2 * kGRows) + int(rank) * kGRows;
    const int wrow0 = nt * kGCols + int(rank) * (kGCols / 2);
    for (int kb = 0; kb < p.k_steps; ++kb, ++it) {
      const int s = it % kGStages;
      const uint32_t ph = uint32_t(it / kGStages) & 1u;
      if (!pair::wait(&sm.empty[s], ph ^ 1u, nullptr, kErrGEmpty, abort_flag)) {
        *issued = it;
        return;
      }
      if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * (kGABytes + kGBBytes));
      const uint32_t full = pair::mapa(&sm.full[s], 0);
#pragma unroll
      for (int at = 0; at < kGAtoms; ++at) {
        pair::tma_load_2d(sm.a[s] + at * kGAtomBytes, &maps.a, full, kb * kGKStep + at * kGAtomK, row0);
        pair::tma_load_2d(sm.b[s] + at * kGAtomBytes, &maps.w, full, kb * kGKStep + at * kGAtomK, wrow0);
      }
    }
  }
  *issued = it;
}

// Descriptor offsets of the K = 16 steps: four inside each 128-byte swizzled
// row, the next atom 16 KB further.
template <int KK>
constexpr uint32_t kGOff = uint32_t(((KK >> 2) * kGAtomBytes + (KK & 3) * 32) >> 4);

template <int... KK>
ICSA_DEV void gemm_issue(uint64_t a_desc, uint64_t b_desc, uint32_t d_tmem, uint32_t acc,
                         std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(256, kGCols, false, false);
  (pair::mma_ss_elect<kGOff<KK>, kGOff<KK>>(d_tmem, a_desc, b_desc, idesc, (KK > 0) ? 1u : acc), ...);
}

// MMA issuer: all 32 lanes of warp 5 of the leader (waits are warp-uniform,
// one elected lane issues each instruction).
ICSA_DEV void gemm_mma(const GemmParams& p, GSmem& sm, uint32_t tmem) {
  volatile int* abort_flag = &sm.abort_flag;
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const uint64_t ad0 = tc::make_sw128_desc(smem_u32(sm.a[0]), 16, 1024);
  const uint64_t bd0 = tc::make_sw128_desc(smem_u32(sm.b[0]), 16, 1024);
  constexpr uint64_t kAStep = uint64_t(kGABytes >> 4), kBStep = uint64_t(kGBBytes >> 4);
  int it = 0, tcount = 0;
  for (int t = cluster; t < p.tiles; t += clusters, ++tcount) {
    const int buf = tcount & 1;
    // the epilogue has read this accumulator's previous tile (two tiles ago)
    if (!pair::warp_wait(&sm.acc_empty[buf], (uint32_t(tcount >> 1) & 1u) ^ 1u, nullptr, kErrGAccEmpty, abort_flag))
      return;
    tc::fence_after_sync();
    const uint32_t d_tmem = tmem + uint32_t(buf) * kGCols;
    for (int kb = 0; kb < p.k_steps; ++kb, ++it) {
      const int s = it % kGStages;
      if (!pair::warp_wait(&sm.full[s], uint32_t(it / kGStages) & 1u, nullptr, kErrGFull, abort_flag)) return;
      tc::fence_after_sync();
      gemm_issue(ad0 + uint64_t(s) * kAStep, bd0 + uint64_t(s) * kBStep, d_tmem, kb > 0 ? 1u : 0u,
                 std::make_integer_sequence<int, 4 * kGAtoms>{});
      pair::commit_both_elect(&sm.empty[s]);
    }
    pair::commit_both_elect(&sm.acc_full[buf]);
  }
}

ICSA_DEV void load_bias32(const __nv_bfloat16* bias, int c0, float (&b)[32]) {
  if (bias == nullptr) {
#pragma unroll
    for (int e = 0; e < 32; ++e) b[e] = 0.f;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(bias + c0);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 u = __ldg(src + v);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      b[v * 8 + 2 * i] = __uint_as_float(w[i] << 16);
      b[v * 8 + 2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
}

// Epilogue warps 0-3 of both CTAs: thread t owns output row t of its CTA's
// 128 rows (TMEM lane t).
ICSA_DEV void gemm_epilogue(const GemmParams& p, GSmem& sm, uint32_t tmem, uint32_t rank) {
  volatile int* abort_flag = &sm.abort_flag;
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t lanes = uint32_t(warp * 32) << 16;
  int tcount = 0;
  for (int t = cluster; t < p.tiles; t += clusters, ++tcount) {
    int mt, nt;
    tile_coords(p, t, mt, nt);
    const int buf = tcount & 1;
    const bool ok = pair::warp_wait(&sm.acc_full[buf], uint32_t(tcount >> 1) & 1u, nullptr, kErrGAccFull, abort_flag);
    tc::fence_after_sync();
    const int r = mt * (2 * kGRows) + int(rank) * kGRows + tid;
    const bool row_ok = ok && r < p.M;
    float* xrow = p.x + size_t(r) * p.ldx;
    const float* grow = p.gate ? p.gate + size_t(r / p.rows_per_batch) * p.gate_bs : nullptr;
#pragma unroll 1
    for (int c = 0; c < kGCols / 32; ++c) {
      uint32_t acc[32];
      tc::tmem_ld32(tmem + lanes + uint32_t(buf * kGCols + c * 32), acc);
      tc::tmem_wait_ld();
      if (c == kGCols / 32 - 1) {
        // every TMEM read of this accumulator is done: the leader may reuse it
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) pair::arrive_cluster(pair::mapa(&sm.acc_empty[buf], 0));
        __syncwarp();
      }
      const int c0 = nt * kGCols + c * 32;
      if (!row_ok || c0 >= p.N) continue;
      float b[32];
      load_bias32(p.bias, c0, b);
      float y[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) y[e] = bf16_round(__fadd_rn(__uint_as_float(acc[e]), b[e]));
      float4* xp = reinterpret_cast<float4*>(xrow + c0);
      if (grow != nullptr) {
        const float4* gp = reinterpret_cast<const float4*>(grow + c0);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float4 xv = xp[v];
          const float4 g = __ldg(gp + v);
          xv.x = __fadd_rn(xv.x, __fmul_rn(y[4 * v + 0], g.x));
          xv.y = __fadd_rn(xv.y, __fmul_rn(y[4 * v + 1], g.y));
          xv.z = __fadd_rn(xv.z, __fmul_rn(y[4 * v + 2], g.z));
          xv.w = __fadd_rn(xv.w, __fmul_rn(y[4 * v + 3], g.w));
          xp[v] = xv;
        }
      } else {
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float4 xv = xp[v];
          xv.x = __fadd_rn(xv.x, y[4 * v + 0]);
          xv.y = __fadd_rn(xv.y, y[4 * v + 1]);
          xv.z = __fadd_rn(xv.z, y[4 * v + 2]);
          xv.w = __fadd_rn(xv.w, y[4 * v + 3]);
          xp[v] = xv;
        }
      }
    }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGThreads, 1)
    linear_residual_kernel(const GemmParams p, const __grid_constant__ GemmMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  GSmem& sm = *reinterpret_cast<GSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = pair::cluster_rank();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], 8);  // one arrival per epilogue warp, both CTAs
    }
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kGMmaWarp) {
    pair::tmem_alloc(&sm.tmem_base, kGTmemCols);
    pair::tmem_relinquish();
  }
  if (warp == kGProducerWarp && lane == 0) {
    prefetch_tensormap(&maps.a);
    prefetch_tensormap(&maps.w);
  }
  tc::fence_before_sync();
  pair::cluster_sync();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  if (warp < 4) {
    gemm_epilogue(p, sm, tmem, rank);
  } else if (warp == kGProducerWarp) {
    if (lane == 0) {
      int issued = 0;
      gemm_producer(p, maps, sm, rank, &issued);
      if (sm.abort_flag && rank == 0) {
        // the leader's full barriers count the bytes of both CTAs: let every
        // copy still in flight land before either CTA releases its memory
        for (int j = max(0, issued - kGStages); j < issued; ++j)
          attn::drain_wait(&sm.full[j % kGStages], uint32_t(j / kGStages) & 1u, nullptr);
      }
    }
  } else if (rank == 0) {
    gemm_mma(p, sm, tmem);
  }
  __syncwarp();
  tc::fence_before_sync();
  pair::cluster_sync();
  if (warp == kGMmaWarp) {
    tc::fence_after_sync();
    pair::tmem_dealloc(tmem, kGTmemCols);
  }
}

}  // namespace

cudaError_t launch_linear_residual(int M, int N, int K, const CUtensorMap& a_map, const CUtensorMap& w_map,
                                   const __nv_bfloat16* bias, float* x, int64_t ldx, const float* gate,
                                   int64_t gate_bs, int rows_per_batch, int num_sms, cudaStream_t stream) {
  GemmParams p;
  p.M = M; p.N = N; p.K = K;
  p.bias = bias; p.x = x; p.ldx = ldx; p.gate = gate; p.gate_bs = gate_bs; p.rows_per_batch = rows_per_batch;
  p.m_tiles = (M + 2 * kGRows - 1) / (2 * kGRows);
  p.n_tiles = (N + kGCols - 1) / kGCols;
  p.tiles = p.m_tiles * p.n_tiles;
  p.k_steps = (K + kGKStep - 1) / kGKStep;
  if (p.tiles == 0) return cudaSuccess;
  GemmMaps maps;
  maps.a = a_map;
  maps.w = w_map;
  const int clusters = std::max(1, std::min(num_sms / 2, p.tiles));
  const size_t smem = sizeof(GSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(linear_residual_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  linear_residual_kernel<<<2 * clusters, kGThreads, smem, stream>>>(p, maps);
  return cudaGetLastError();
}

ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_gemm)

}  // namespace icsa
