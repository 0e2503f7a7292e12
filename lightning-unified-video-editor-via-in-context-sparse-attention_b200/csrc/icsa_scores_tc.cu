// Block-score GEMMs of the selection stage on the tensor cores:
//
//   compressed scores (editing_sparse_attention.py:58-59)
//     scores[bh, i, j] = (Qc[bh, i, :] . Kc[bh, j, :]) / sqrt(D)
//   per-sparse-block scores (tilelang_host.py:172)
//     blockscore[bh, r, j] = QC[bh, order[num_flat + r], :] . KC[bh, j, :]
//
// The operands hold bf16 values: the bf16 block sums, and the pooled means of
// bf16 inputs (or of f32 inputs whose compressed attention runs in bf16),
// which the pool stage rounds to bf16.  Every product of two bf16 values is
// exact in fp32, so a tcgen05 kind::f16 MMA with an fp32 accumulator computes
// the same dot products as fp32 FMAs up to the order of the additions.  The
// selections are defined on these fp32 keys as the GPU computes them (ties to
// the lower index), so the summation order changes no contract, only low
// bits of the keys.
//
// One CTA: 128 A rows x 128 B rows, 256 threads.
//   1. all threads load their share of both operands (f32 rows are converted
//      to bf16; bf16 rows are copied) into shared memory in the
//      128-byte-swizzled K-major layout; A rows may be gathered through an
//      index table;
//   2. one elected lane of warp 0 issues D/16 MMAs (M = 128, N = 128, K = 16)
//      into 128 TMEM columns and commits them to an mbarrier;
//   3. warps w and w + 4 read TMEM lanes [32 (w % 4), +32) (their A rows),
//      alternate 32-column chunks, divide by the divisor if one is given, and
//      write the tile through a shared-memory transpose so that each store
//      instruction covers 128 contiguous bytes of one output row.
// Three CTAs fit on an SM (65 KB of shared memory and 128 TMEM columns each).
#include "icsa_kernels.cuh"
#include "icsa_tcgen05.cuh"

#include <cstring>
#include <utility>

namespace icsa {

namespace {

constexpr int kTM = 128;       // A rows per CTA (TMEM lanes)
// B rows per CTA (TMEM columns).  128 rather than 256: twice the CTAs and
// half the epilogue per CTA measured 4-25 us faster for the scores GEMM
// (5-40 heads of 480p), the extra reads of A coming from L2.
constexpr int kTN = 128;
constexpr int kThreads = 256;  // warps w and w + 4 share TMEM lanes [32 (w % 4), +32)
constexpr int kErrScoresMma = 0x201;
constexpr int kErrScoresDrain = 0x202;

constexpr int kStageBytes = 8 * 32 * 33 * 4;  // the epilogue's transpose buffers

template <int D>
struct ScoresSmem {
  // D/64 chunks of 64 features; a row of a chunk is 128 bytes (64 bf16)
  uint8_t a[D / 64][kTM * 128];
  uint8_t b[D / 64][kTN * 128];
  // the transpose buffers reuse a and b; this pads them where they are smaller
  uint8_t pad[(D / 64) * (kTM + kTN) * 128 >= kStageBytes ? 16 : kStageBytes - (D / 64) * (kTM + kTN) * 128];
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

// One operand: row r of head bh is row (idx ? idx[bh * idx_bh + r] : r) of
// the [rows_total, D] matrix at base + bh * bh_stride (elements); rows at or
// beyond `rows` are zero.
struct Operand {
  const void* base;
  int f32;              // 1: f32 elements holding bf16 values, 0: bf16
  long long bh_stride;  // elements between heads
  const int* idx;       // optional row gather table
  long long idx_bh;     // entries between heads of idx
  int rows;
};

struct GemmArgs {
  Operand a, b;
  float* out;           // out[bh * out_bh + r * ld + j]
  long long out_bh;
  int ld;
  float div;            // > 0: each value is divided by it (IEEE division)
  int* err;
};

// Rows [row0, row0 + R) of an operand, as bf16 in the swizzled K-major layout:
// feature k of row r lives in chunk k / 64 at byte
// r * 128 + ((k % 64) / 8 ^ r % 8) * 16 + (k % 8) * 2.
// The loads of a batch of kBatch 16-byte units per thread are all issued
// before any is converted or stored, so that a thread has kBatch (bf16) or
// 2 kBatch (f32) loads in flight instead of one.
constexpr int kBatch = 8;

ICSA_DEV void store_unit(uint8_t* chunk0, int chunk_bytes, int r, int c8, uint4 w) {
  const int chunk = c8 >> 3, unit = c8 & 7;
  *reinterpret_cast<uint4*>(chunk0 + chunk * chunk_bytes + r * 128 + ((unit ^ (r & 7)) << 4)) = w;
}

template <int D, int R>
ICSA_DEV void stage_operand(uint8_t (*dst)[R * 128], const Operand& o, int bh, int row0) {
  constexpr int kUnits = D / 8;                   // 16-byte units of bf16 per row
  constexpr int kPerThread = R * kUnits / kThreads;
  constexpr int kB = kPerThread < kBatch ? kPerThread : kBatch;
  static_assert(kPerThread % kB == 0, "whole batches per thread");
  // unit u = threadIdx.x + kThreads * i: consecutive threads read consecutive
  // units of a row
  const long long head = bh * o.bh_stride;
#pragma unroll 1
  for (int i0 = 0; i0 < kPerThread; i0 += kB) {
    long long src[kB];
    bool live[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int u = threadIdx.x + kThreads * (i0 + i);
      const int r = u / kUnits, c8 = u % kUnits;
      live[i] = row0 + r < o.rows;
      const long long row = !live[i] ? 0 : (o.idx ? o.idx[bh * o.idx_bh + row0 + r] : row0 + r);
      src[i] = head + row * D + c8 * 8;
    }
    if (o.f32) {
      const float* base = static_cast<const float*>(o.base);
      float4 x[kB][2];
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const float4* s = reinterpret_cast<const float4*>(base + src[i]);
        x[i][0] = live[i] ? __ldg(s) : make_float4(0.f, 0.f, 0.f, 0.f);
        x[i][1] = live[i] ? __ldg(s + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int u = threadIdx.x + kThreads * (i0 + i);
        store_unit(dst[0], R * 128, u / kUnits, u % kUnits,
                   make_uint4(pack_bf16x2(x[i][0].x, x[i][0].y), pack_bf16x2(x[i][0].z, x[i][0].w),
                              pack_bf16x2(x[i][1].x, x[i][1].y), pack_bf16x2(x[i][1].z, x[i][1].w)));
      }
    } else {
      const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(o.base);
      uint4 x[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i)
        x[i] = live[i] ? __ldg(reinterpret_cast<const uint4*>(base + src[i])) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        const int u = threadIdx.x + kThreads * (i0 + i);
        store_unit(dst[0], R * 128, u / kUnits, u % kUnits, x[i]);
      }
    }
  }
}

// K step kk: 16 features = 32 bytes inside the 128-byte row, the next chunk
// of 64 features R * 128 bytes further (descriptor units of 16 bytes).
template <int R, int KK>
constexpr uint32_t kKOff = uint32_t(((KK >> 2) * R * 128 + (KK & 3) * 32) >> 4);

template <int... KK>
ICSA_DEV void issue_scores(uint64_t a_desc, uint64_t b_desc, uint32_t d_tmem, std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(kTM, kTN, false, false);
  (tc::mma_bf16_ss_elect<kKOff<kTM, KK>, kKOff<kTN, KK>>(d_tmem, a_desc, b_desc, idesc, KK > 0 ? 1u : 0u), ...);
}

template <int D>
__global__ void __launch_bounds__(kThreads) block_gemm_kernel(const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  // SW128 operands need 1024-byte alignment
  ScoresSmem<D>& sm = *reinterpret_cast<ScoresSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kTM, j0 = blockIdx.x * kTN;

  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem_base, kTN);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    mbar_init(&sm.done, 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  wait_prior_grid();  // the operands are the previous kernels' outputs
  stage_operand<D, kTM>(sm.a, g.a, bh, i0);
  stage_operand<D, kTN>(sm.b, g.b, bh, j0);
  // the generic-proxy stores must be visible to the tensor core's reads
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  if (warp == 0) {
    const uint64_t ad = tc::make_sw128_desc(smem_u32(sm.a[0]), 16, 1024);
    const uint64_t bd = tc::make_sw128_desc(smem_u32(sm.b[0]), 16, 1024);
    issue_scores(ad, bd, tmem, std::make_integer_sequence<int, D / 16>{});
    tc::mma_commit_elect(&sm.done);
  }
  const bool ok = mbar_wait(&sm.done, 0, g.err, kErrScoresMma, &sm.abort_flag);
  __syncwarp();
  if (__all_sync(0xffffffffu, ok)) {
    tc::fence_after_sync();
    // transpose buffer of this warp, over the (now idle) operands and the
    // padding after them
    float(*stg)[33] = reinterpret_cast<float(*)[33]>(sm.a[0] + warp * 32 * 33 * sizeof(float));
    float* out = g.out + bh * g.out_bh;
    const int quarter = warp & 3;  // TMEM lanes (A rows) this warp may read
    const uint32_t lanes = uint32_t(quarter * 32) << 16;
#pragma unroll 1
    for (int c = warp >> 2; c < kTN / 32; c += kThreads / 128) {
      if (j0 + 32 * c >= g.b.rows) break;  // warp-uniform
      uint32_t r[32];
      tc::tmem_ld32(tmem + lanes + uint32_t(32 * c), r);
      tc::tmem_wait_ld();
      if (g.div > 0.f) {
#pragma unroll
        for (int e = 0; e < 32; ++e) stg[lane][e] = __uint_as_float(r[e]) / g.div;
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) stg[lane][e] = __uint_as_float(r[e]);
      }
      __syncwarp();
      const int col = j0 + 32 * c + lane;
#pragma unroll 4
      for (int rr = 0; rr < 32; ++rr) {
        const int row = i0 + quarter * 32 + rr;
        if (row < g.a.rows && col < g.b.rows) out[size_t(row) * g.ld + col] = stg[rr][lane];
      }
      __syncwarp();
    }
  } else if (threadIdx.x == 0) {
    // the MMAs may still be running: give them a bounded time to finish
    // before their TMEM columns are released
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(&sm.done, 0))
      if (global_timer_ns() - t0 > 1000000000ull) {
        report_error(g.err, kErrScoresDrain);
        break;
      }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kTN);
}

template <int D>
cudaError_t launch_gemm(const GemmArgs& g, int BH, cudaStream_t stream) {
  if (g.a.rows <= 0 || g.b.rows <= 0 || BH <= 0) return cudaSuccess;
  const size_t smem = sizeof(ScoresSmem<D>) + 1024;  // + alignment slack
  const cudaError_t e =
      cudaFuncSetAttribute(block_gemm_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((g.b.rows + kTN - 1) / kTN, (g.a.rows + kTM - 1) / kTM, BH);
  return launch_chained(block_gemm_kernel<D>, grid, dim3(kThreads), smem, stream, g);
}

cudaError_t launch_gemm(const GemmArgs& g, int D, int BH, cudaStream_t stream) {
  if (D == 128) return launch_gemm<128>(g, BH, stream);
  if (D == 64) return launch_gemm<64>(g, BH, stream);
  return cudaErrorInvalidValue;
}


// ---------------------------------------------------------------------------
// out_c on the tensor cores (editing_sparse_attention.py:60-63):
//
//   out_c[bh, i, :] = sum_j P[i, j] Vc[bh, j, :],  P = exp(s - m_i) / l_i
//
// with P computed exactly as the CUDA-core kernel computes it (fp32,
// 2^((s - m) log2 e) times 1/l).  P is split into two bf16 terms,
// hi = bf16(P) and lo = bf16(P - hi), and both are multiplied by the bf16
// values of Vc (the pooled means of bf16 values), so the products are exact
// and the result carries P to about 16 bits (relative error below 2^-16 per
// term) with fp32 accumulation.
//
// One CTA: 128 rows of one (b, h), 256 threads, keys in chunks of 64 through
// two shared-memory stages {P_hi, P_lo, Vc}:
//   * threads 0-127 (one row each) turn their row's 64 scores into P_hi/P_lo
//     rows of the 128-byte-swizzled K-major A operands, with the next chunk's
//     scores already loaded into registers;
//   * threads 128-255 convert the chunk's 64 rows of Vc into the swizzled
//     MN-major B operand (64 keys x D features);
//   * after a barrier one elected lane issues 2 x 4 MMAs (M = 128, N = D,
//     K = 16 keys) into the accumulator and commits them to the stage's
//     mbarrier, which releases the stage two chunks later.
// ---------------------------------------------------------------------------
constexpr int kOKeys = 64;  // keys per chunk
constexpr int kErrOutcMma = 0x203;

template <int D>
struct OutcSmem {
  uint8_t phi[2][128 * 128];       // [stage][row][64 keys bf16], swizzled
  uint8_t plo[2][128 * 128];
  uint8_t v[2][D / 64][kOKeys * 128];  // [stage][d chunk][key][64 d bf16], swizzled
  uint64_t mma_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

template <int D, int... KK>
ICSA_DEV void issue_outc(uint64_t hi_desc, uint64_t lo_desc, uint64_t v_desc, uint32_t d_tmem, uint32_t acc,
                         std::integer_sequence<int, KK...>) {
  constexpr uint32_t idesc = tc::make_idesc_bf16(128, D, false, true);
  // A: 16 keys = 32 bytes along the swizzled row; B: 16 keys = 16 rows of 128 B
  (tc::mma_bf16_ss_elect<uint32_t(KK * 2), uint32_t(KK * 128)>(d_tmem, hi_desc, v_desc, idesc,
                                                               (KK > 0 || acc) ? 1u : 0u), ...);
  (tc::mma_bf16_ss_elect<uint32_t(KK * 2), uint32_t(KK * 128)>(d_tmem, lo_desc, v_desc, idesc, 1u), ...);
}

template <int D>
__global__ void __launch_bounds__(256) outc_tc_kernel(SelectParams p) {
  extern __shared__ uint8_t smem_raw[];
  OutcSmem<D>& sm = *reinterpret_cast<OutcSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int i0 = blockIdx.x * 128;
  const int NB = p.NB;
  const int n_chunks = (NB + kOKeys - 1) / kOKeys;
  constexpr float kLog2e = 1.4426950408889634f;

  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem_base, D);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&sm.mma_done[0], 1);
    mbar_init(&sm.mma_done[1], 1);
    sm.abort_flag = 0;
    fence_mbarrier_init();
  }
  // P rows: thread tid < 128 owns row i0 + tid
  const bool prow = tid < 128;
  const int i = i0 + (tid & 127);
  const bool row_ok = prow && i < NB;
  float m = 0.f, il = 0.f;
  if (row_ok) {
    m = p.rowmax[size_t(bh) * NB + i] * kLog2e;
    il = 1.0f / p.rowsum[size_t(bh) * NB + i];
  }
  const float* srow = p.scores + (size_t(bh) * NB + (row_ok ? i : 0)) * NB;
  const float* V = p.vmean + size_t(bh) * NB * D;
  const bool vec = (NB & 3) == 0;  // every row starts on a 16-byte boundary
  float4 raw[kOKeys / 4];          // this row's scores of the chunk being converted
  auto load_scores = [&](int c) {
    const int j0 = c * kOKeys;
#pragma unroll
    for (int e = 0; e < kOKeys / 4; ++e) {
      const int j = j0 + 4 * e;
      if (vec && row_ok && j + 3 < NB) {
        raw[e] = __ldg(reinterpret_cast<const float4*>(srow + j));
      } else {
        // ragged end, or rows NB floats apart that do not keep 16-byte alignment
        float t[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) t[q] = (row_ok && j + q < NB) ? srow[j + q] : 0.f;
        raw[e] = make_float4(t[0], t[1], t[2], t[3]);
      }
    }
  };
  if (prow) load_scores(0);
  __syncthreads();  // barriers initialised, TMEM allocated
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  bool ok = true;
#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c & 1;
    const int j0 = c * kOKeys;
    // the stage was last read by the MMAs of chunk c - 2
    if (c >= 2 && ok) ok = mbar_wait(&sm.mma_done[st], uint32_t((c - 2) >> 1) & 1u, p.err, kErrOutcMma,
                                     &sm.abort_flag);
    if (prow) {
      // raw holds chunk c; P = 2^(s log2e - m) / l, split into bf16 hi + lo
      uint8_t* hrow = sm.phi[st] + tid * 128;
      uint8_t* lrow = sm.plo[st] + tid * 128;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float pv[8];
        const float4 a = raw[2 * u], b = raw[2 * u + 1];
        const float sv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int j = j0 + 8 * u + q;
          float ex;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ex) : "f"(fmaf(sv[q], kLog2e, -m)));
          pv[q] = (row_ok && j < NB) ? ex * il : 0.f;
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __nv_bfloat16 h0 = __float2bfloat16_rn(pv[2 * q]), h1 = __float2bfloat16_rn(pv[2 * q + 1]);
          hi[q] = uint32_t(__bfloat16_as_ushort(h0)) | (uint32_t(__bfloat16_as_ushort(h1)) << 16);
          lo[q] = pack_bf16x2(pv[2 * q] - __bfloat162float(h0), pv[2 * q + 1] - __bfloat162float(h1));
        }
        const int off = (u ^ (tid & 7)) << 4;
        *reinterpret_cast<uint4*>(hrow + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(lrow + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      if (c + 1 < n_chunks) load_scores(c + 1);
    } else {
      // Vc rows j0 .. j0 + 63: unit (key k, 8 features from d8 * 8)
      constexpr int kUnits = kOKeys * D / 8;
      const int t = tid - 128;
#pragma unroll 4
      for (int u = t; u < kUnits; u += 128) {
        const int k = u / (D / 8), d8 = u % (D / 8);
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (j0 + k < NB) {
          const float4* src = reinterpret_cast<const float4*>(V + size_t(j0 + k) * D + d8 * 8);
          const float4 x0 = __ldg(src), x1 = __ldg(src + 1);
          w = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                         pack_bf16x2(x1.z, x1.w));
        }
        *reinterpret_cast<uint4*>(sm.v[st][d8 >> 3] + k * 128 + (((d8 & 7) ^ (k & 7)) << 4)) = w;
      }
    }
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0 && __all_sync(0xffffffffu, ok) && !sm.abort_flag) {
      tc::fence_after_sync();
      const uint64_t hd = tc::make_sw128_desc(smem_u32(sm.phi[st]), 16, 1024);
      const uint64_t ld = tc::make_sw128_desc(smem_u32(sm.plo[st]), 16, 1024);
      const uint64_t vd = tc::make_sw128_desc(smem_u32(sm.v[st][0]), kOKeys * 128, 1024);
      issue_outc<D>(hd, ld, vd, tmem, c > 0 ? 1u : 0u, std::make_integer_sequence<int, kOKeys / 16>{});
      tc::mma_commit_elect(&sm.mma_done[st]);
    }
  }
  // the last chunk's commit covers every MMA issued before it
  const int last = n_chunks - 1;
  if (ok) ok = mbar_wait(&sm.mma_done[last & 1], uint32_t(last >> 1) & 1u, p.err, kErrOutcMma, &sm.abort_flag);
  __syncwarp();
  if (warp < 4 && __all_sync(0xffffffffu, ok)) {
    tc::fence_after_sync();
    const int row = i0 + warp * 32 + lane;
    float* O = p.outc + (size_t(bh) * NB + row) * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      tc::tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(32 * c), r);
      tc::tmem_wait_ld();
      if (row < NB) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(O + 32 * c + e) = make_float4(
              __uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
      }
    }
  } else if (!ok && tid == 0) {
    // give MMAs still in flight a bounded time before their columns go
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(&sm.mma_done[last & 1], uint32_t(last >> 1) & 1u))
      if (global_timer_ns() - t0 > 1000000000ull) {
        report_error(p.err, kErrScoresDrain);
        break;
      }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, D);
}

template <int D>
cudaError_t launch_outc_tc_d(const SelectParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(OutcSmem<D>) + 1024;
  const cudaError_t e = cudaFuncSetAttribute(outc_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((p.NB + 127) / 128, p.B * p.H);
  outc_tc_kernel<D><<<grid, 256, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_scores_tc(const SelectParams& p, cudaStream_t stream) {
  GemmArgs g;
  std::memset(&g, 0, sizeof(g));
  g.a = Operand{p.qmean, 1, (long long)p.NB * p.D, nullptr, 0, p.NB};
  g.b = Operand{p.kmean, 1, (long long)p.NB * p.D, nullptr, 0, p.NB};
  g.out = p.scores;
  g.out_bh = (long long)p.NB * p.NB;
  g.ld = p.NB;
  g.div = p.inv_sqrt_d_div;
  g.err = p.err;
  return launch_gemm(g, p.D, p.B * p.H, stream);
}

cudaError_t launch_blockscore_tc(const SelectParams& p, cudaStream_t stream) {
  GemmArgs g;
  std::memset(&g, 0, sizeof(g));
  // the sparse query blocks, in the order of the sharpness split
  g.a = Operand{p.qsum, 0, (long long)p.NB * p.D, p.order + p.num_flat, p.NB, p.n_sparse};
  g.b = Operand{p.kc, 0, (long long)p.nkv_pad * p.D, nullptr, 0, p.nkv};
  g.out = p.blockscore;
  g.out_bh = (long long)p.n_sparse * p.nkv;
  g.ld = p.nkv;
  g.div = 0.f;
  g.err = p.err;
  return launch_gemm(g, p.D, p.B * p.H, stream);
}

cudaError_t launch_outc_tc(const SelectParams& p, cudaStream_t stream) {
  if (p.NB <= 0 || p.B * p.H <= 0) return cudaSuccess;
  if (p.D == 128) return launch_outc_tc_d<128>(p, stream);
  if (p.D == 64) return launch_outc_tc_d<64>(p, stream);
  return cudaErrorInvalidValue;
}

ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_scores)

}  // namespace icsa
