// Stage 2: compressed (block-level) attention and all block selections.
//
// Restates editing_sparse_attention.py:58-64,113-172 and the host top-k of
// the sparse backend (tilelang_host.py:170-173):
//   scores  = Qc . Kc^T / sqrt(D)   over all NB x NB block pairs (fp32)
//   P       = softmax(scores) per row; out_c = P . Vc
//   colsum  = sum of P[target rows, source columns]      -> top-K source blocks
//   sharp   = sum of the k_sparsity largest P[row, target columns]
//             -> stable descending order; the first num_flat blocks are "flat"
//   per sparse query block: fp32 QC . KC^T over the extended KV blocks
//             -> top_k blocks for exact attention.
// Every selection is a total order on (value desc, index asc), so ties go to
// the lower index and the result is deterministic.  All reductions run in a
// fixed order (no atomics), so repeated calls give identical bits.
#include "icsa_kernels.cuh"
#include "icsa_sort.cuh"

#include <math.h>

namespace icsa {

namespace {

// ---------------------------------------------------------------------------
// scores[bh, i, j] = dot(qmean[bh, i], kmean[bh, j]) / sqrt(D)
// 128x128 output tile per CTA, 256 threads, 8x8 outputs per thread (rows and
// columns split into two groups of 4, 64 apart, so that the float4 reads of
// shared memory are conflict-free).  Every output accumulates over k in
// increasing order with fmaf-rounded FMAs (two outputs per f32x2
// instruction), then divides by sqrt(D).
// ---------------------------------------------------------------------------
constexpr int kGT = 128;  // GEMM tile
constexpr int kGK = 8;    // GEMM k-chunk

// Two independent fp32 FMAs in one packed instruction (sm_100 f32x2):
// x = a0 * b0 + x, y = a1 * b1 + y, each rounded as fmaf rounds it, so every
// output still accumulates over k in the same order with the same bits.
ICSA_DEV void fma_x2(float& x, float& y, float a0, float a1, float b0, float b1) {
  asm("{.reg .b64 a, b, c;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%0, %1};\n\t"
      "fma.rn.f32x2 c, a, b, c;\n\tmov.b64 {%0, %1}, c;}"
      : "+f"(x), "+f"(y)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__global__ void __launch_bounds__(256) scores_kernel(SelectParams p) {
  __shared__ __align__(16) float As[kGK][kGT + 4];
  __shared__ __align__(16) float Bs[kGK][kGT + 4];
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kGT, j0 = blockIdx.x * kGT;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const float* A = p.qmean + size_t(bh) * p.NB * p.D;
  const float* Bm = p.kmean + size_t(bh) * p.NB * p.D;
  const int lr = threadIdx.x >> 1, lk = (threadIdx.x & 1) * 4;  // loader: row, first k of a float4
  const bool ra = i0 + lr < p.NB, rb = j0 + lr < p.NB;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  // the next k-chunk is loaded into registers while the current one is used
  float4 va = ra ? *reinterpret_cast<const float4*>(A + size_t(i0 + lr) * p.D + lk) : z4;
  float4 vb = rb ? *reinterpret_cast<const float4*>(Bm + size_t(j0 + lr) * p.D + lk) : z4;
  float acc[8][8] = {};
  for (int k0 = 0; k0 < p.D; k0 += kGK) {
    As[lk + 0][lr] = va.x; As[lk + 1][lr] = va.y; As[lk + 2][lr] = va.z; As[lk + 3][lr] = va.w;
    Bs[lk + 0][lr] = vb.x; Bs[lk + 1][lr] = vb.y; Bs[lk + 2][lr] = vb.z; Bs[lk + 3][lr] = vb.w;
    __syncthreads();
    if (k0 + kGK < p.D) {
      va = ra ? *reinterpret_cast<const float4*>(A + size_t(i0 + lr) * p.D + k0 + kGK + lk) : z4;
      vb = rb ? *reinterpret_cast<const float4*>(Bm + size_t(j0 + lr) * p.D + k0 + kGK + lk) : z4;
    }
#pragma unroll
    for (int c = 0; c < kGK; ++c) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[c][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[c][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[c][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[c][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int w = 0; w < 8; w += 2) fma_x2(acc[u][w], acc[u][w + 1], a[u], a[u], b[w], b[w + 1]);
    }
    __syncthreads();
  }
  float* S = p.scores + size_t(bh) * p.NB * p.NB;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int i = i0 + (u < 4 ? ty * 4 + u : 64 + ty * 4 + u - 4);
    if (i >= p.NB) continue;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int j = j0 + (w < 4 ? tx * 4 + w : 64 + tx * 4 + w - 4);
      if (j < p.NB) S[size_t(i) * p.NB + j] = acc[u][w] / p.inv_sqrt_d_div;
    }
  }
}

// ---------------------------------------------------------------------------
// Per row: softmax statistics and the sharpness key.  One warp per row; the
// k_sparsity-th largest target-column score is found by a radix select over
// order-preserving keys, and the sharpness is the sum of the probabilities
// above it plus the remaining ties at it (the sum of the k_sparsity largest).
// ---------------------------------------------------------------------------
ICSA_DEV float order_key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// exp(x) and a / b for the softmax statistics: the fast intrinsics (relative
// error about 2^-21) for the row statistics of the tensor-core scores, whose
// low bits are the GPU's own already; the library functions otherwise.
template <bool kFast>
ICSA_DEV float stat_exp(float x) {
  if constexpr (kFast) return __expf(x);
  else return expf(x);
}
template <bool kFast>
ICSA_DEV float stat_div(float a, float b) {
  if constexpr (kFast) return __fdividef(a, b);
  else return a / b;
}

template <bool kFast>
__global__ void rowstats_kernel(SelectParams p, int warps, int stride) {
  extern __shared__ uint32_t sh_rs[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.y;
  const int i = blockIdx.x * warps + warp;
  wait_prior_grid();
  if (i >= p.NB) return;
  const float* S = p.scores + (size_t(bh) * p.NB + i) * p.NB;
  float m = -INFINITY;
  for (int j = lane; j < p.NB; j += 32) m = fmaxf(m, S[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.f;
  for (int j = lane; j < p.NB; j += 32) l += stat_exp<kFast>(S[j] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);

  float sharp = 0.f;
  const int kk = min(p.k_sparsity, p.n_t);
  if (kk > 0) {
    uint32_t* keys = sh_rs + size_t(warp) * stride;
    uint32_t* hist = sh_rs + size_t(warps) * stride + warp * 256;
    for (int j = lane; j < p.n_t; j += 32) keys[j] = float_order_key(S[j]);
    __syncwarp();
    int n_gt = 0;
    const uint32_t kth = warp_kth_largest(keys, p.n_t, kk, hist, &n_gt);
    float acc = 0.f;
    for (int j = lane; j < p.n_t; j += 32)
      if (keys[j] > kth) acc += stat_div<kFast>(stat_exp<kFast>(S[j] - m), l);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    sharp = acc + float(kk - n_gt) * stat_div<kFast>(stat_exp<kFast>(order_key_to_float(kth) - m), l);
  }
  if (lane == 0) {
    p.rowmax[size_t(bh) * p.NB + i] = m;
    p.rowsum[size_t(bh) * p.NB + i] = l;
    p.sharp[size_t(bh) * p.NB + i] = sharp;
  }
}

// ---------------------------------------------------------------------------
// out_c[bh, i, :] = sum_j P[i, j] * vmean[bh, j, :],  P = exp(s - m) / l.
// A CTA owns 64 rows and all D columns, so each probability is computed once
// (2^((s - m) log2 e) times 1/l); chunks of 32 columns of P and rows of V are
// staged in shared memory.  256 threads, 4 rows x D/16 columns per thread.
// ---------------------------------------------------------------------------
constexpr int kOR = 64;   // rows per CTA
constexpr int kOJ = 32;   // j per chunk

ICSA_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(256) outc_kernel(SelectParams p) {
  constexpr int kCW = D / 16;  // columns per thread: D/64 groups of 4, 64 apart
  __shared__ __align__(16) float Ps[kOJ][kOR + 4];
  __shared__ __align__(16) float Vs[kOJ][D + 4];
  __shared__ float sm[kOR], sl[kOR];
  const int bh = blockIdx.y;
  const int i0 = blockIdx.x * kOR;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const float* S = p.scores + size_t(bh) * p.NB * p.NB;
  const float* V = p.vmean + size_t(bh) * p.NB * D;
  constexpr float kLog2e = 1.4426950408889634f;
  if (threadIdx.x < kOR) {
    const int i = i0 + threadIdx.x;
    sm[threadIdx.x] = (i < p.NB) ? p.rowmax[size_t(bh) * p.NB + i] * kLog2e : 0.f;
    sl[threadIdx.x] = (i < p.NB) ? 1.0f / p.rowsum[size_t(bh) * p.NB + i] : 0.f;
  }
  __syncthreads();
  const int pr = threadIdx.x >> 2, pc = (threadIdx.x & 3) * 8;  // P loader: row, first of 8 columns
  constexpr int kVL = kOJ * D / 4 / 256;                          // float4 of V per thread and chunk
  const int i = i0 + pr;
  // the scores and V rows of the next chunk are loaded into registers while
  // the current chunk is used
  float sraw[8];
  float4 vr[kVL];
  auto fetch = [&](int j0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = j0 + pc + e;
      sraw[e] = (i < p.NB && j < p.NB) ? S[size_t(i) * p.NB + j] : 0.f;
    }
#pragma unroll
    for (int t = 0; t < kVL; ++t) {
      const int e = threadIdx.x + t * 256;
      const int jr = e / (D / 4), dc = (e % (D / 4)) * 4;
      vr[t] = (j0 + jr < p.NB) ? *reinterpret_cast<const float4*>(V + size_t(j0 + jr) * D + dc)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float acc[4][kCW] = {};
  fetch(0);
  for (int j0 = 0; j0 < p.NB; j0 += kOJ) {
    {
      const float m = sm[pr], il = sl[pr];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + pc + e;
        Ps[pc + e][pr] = (i < p.NB && j < p.NB) ? fast_exp2(fmaf(sraw[e], kLog2e, -m)) * il : 0.f;
      }
    }
#pragma unroll
    for (int t = 0; t < kVL; ++t) {
      const int e = threadIdx.x + t * 256;
      *reinterpret_cast<float4*>(&Vs[e / (D / 4)][(e % (D / 4)) * 4]) = vr[t];
    }
    __syncthreads();
    if (j0 + kOJ < p.NB) fetch(j0 + kOJ);
#pragma unroll 8
    for (int c = 0; c < kOJ; ++c) {
      const float4 a = *reinterpret_cast<const float4*>(&Ps[c][ty * 4]);
      float b[kCW];
#pragma unroll
      for (int g = 0; g < kCW / 4; ++g) {
        const float4 v = *reinterpret_cast<const float4*>(&Vs[c][g * 64 + tx * 4]);
        b[4 * g] = v.x; b[4 * g + 1] = v.y; b[4 * g + 2] = v.z; b[4 * g + 3] = v.w;
      }
      const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < kCW; w += 2) fma_x2(acc[u][w], acc[u][w + 1], av[u], av[u], b[w], b[w + 1]);
    }
    __syncthreads();
  }
  float* O = p.outc + size_t(bh) * p.NB * D;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty * 4 + u;
    if (i >= p.NB) continue;
#pragma unroll
    for (int g = 0; g < kCW / 4; ++g) {
      const int d = g * 64 + tx * 4;
      *reinterpret_cast<float4*>(O + size_t(i) * D + d) =
          make_float4(acc[u][4 * g], acc[u][4 * g + 1], acc[u][4 * g + 2], acc[u][4 * g + 3]);
    }
  }
}

// ---------------------------------------------------------------------------
// colsum[bh, j] = sum over target rows i < n_t of P[i, n_t + j].  A CTA owns
// 32 columns; its 8 row groups each add every 8th row in increasing order and
// the 8 partial sums are combined in a fixed order (deterministic).
// ---------------------------------------------------------------------------
template <bool kFast>
__global__ void colsum_kernel(SelectParams p) {
  __shared__ float part[8][33];
  const int bh = blockIdx.y;
  const int c = threadIdx.x, g = threadIdx.y;
  const int j = blockIdx.x * 32 + c;
  const float* M = p.rowmax + size_t(bh) * p.NB;
  const float* L = p.rowsum + size_t(bh) * p.NB;
  wait_prior_grid();
  float acc = 0.f;
  if (j < p.n_s) {
    const float* S = p.scores + size_t(bh) * p.NB * p.NB + p.n_t + j;
    // this group's rows g, g + 8, ... in increasing order; eight rows' loads
    // are issued before their terms are added
    int i = g;
    for (; i + 56 < p.n_t; i += 64) {
      float s[8], mm[8], ll[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        s[u] = S[size_t(i + 8 * u) * p.NB];
        mm[u] = M[i + 8 * u];
        ll[u] = L[i + 8 * u];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc += stat_div<kFast>(stat_exp<kFast>(s[u] - mm[u]), ll[u]);
    }
    for (; i < p.n_t; i += 8) acc += stat_div<kFast>(stat_exp<kFast>(S[size_t(i) * p.NB] - M[i]), L[i]);
  }
  part[g][c] = acc;
  __syncthreads();
  if (g == 0 && j < p.n_s) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k][c];
    p.colsum[size_t(bh) * p.n_s + j] = t;
  }
}

}  // namespace

cudaError_t launch_compressed_scores(const SelectParams& p, cudaStream_t stream) {
  const int BH = p.B * p.H;
  cudaError_t e;
  if (p.means_bf16 && (p.D == 64 || p.D == 128)) {
    e = launch_scores_tc(p, stream);
  } else {
    // f32 means: fp32 FMAs on the CUDA cores
    dim3 g1((p.NB + kGT - 1) / kGT, (p.NB + kGT - 1) / kGT, BH);
    scores_kernel<<<g1, 256, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;

  const int stride = p.n_t > 0 ? p.n_t : 1;
  int warps = 8;
  auto rs_smem = [&](int w) { return size_t(w) * stride * sizeof(uint32_t) + size_t(w) * 256 * sizeof(uint32_t); };
  while (warps > 1 && rs_smem(warps) > 96 * 1024) warps >>= 1;
  const size_t smem = rs_smem(warps);
  if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
  const bool fast = p.means_bf16 && (p.D == 64 || p.D == 128);  // the tensor-core scores
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(fast ? rowstats_kernel<true> : rowstats_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  dim3 g2((p.NB + warps - 1) / warps, BH);
  return launch_chained(fast ? rowstats_kernel<true> : rowstats_kernel<false>, g2, dim3(warps * 32), smem, stream,
                        p, warps, stride);
}

cudaError_t launch_outc(const SelectParams& p, cudaStream_t stream) {
  if (p.vmean_bf16 && (p.D == 64 || p.D == 128)) return launch_outc_tc(p, stream);
  // f32 means: fp32 FMAs on the CUDA cores
  dim3 g3((p.NB + kOR - 1) / kOR, p.B * p.H);
  if (p.D == 128) outc_kernel<128><<<g3, 256, 0, stream>>>(p);
  else if (p.D == 64) outc_kernel<64><<<g3, 256, 0, stream>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_colsum(const SelectParams& p, cudaStream_t stream) {
  if (p.n_s <= 0) return cudaSuccess;
  dim3 g4((p.n_s + 31) / 32, p.B * p.H);
  // (the fast forms measured slower here: 8.9 -> 12.9 us at 5 heads)
  return launch_chained(colsum_kernel<false>, g4, dim3(32, 8), 0, stream, p);
}

}  // namespace icsa
