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
// 64x64 output tile per CTA, 256 threads, 4x4 outputs per thread.
// ---------------------------------------------------------------------------
constexpr int kGT = 64;   // GEMM tile
constexpr int kGK = 16;   // GEMM k-chunk

__global__ void __launch_bounds__(256) scores_kernel(SelectParams p) {
  __shared__ float As[kGK][kGT + 4];
  __shared__ float Bs[kGK][kGT + 4];
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kGT, j0 = blockIdx.x * kGT;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const float* A = p.qmean + size_t(bh) * p.NB * p.D;
  const float* Bm = p.kmean + size_t(bh) * p.NB * p.D;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.D; k0 += kGK) {
    for (int e = threadIdx.x; e < kGT * kGK; e += 256) {
      const int r = e / kGK, c = e % kGK;
      As[c][r] = (i0 + r < p.NB) ? A[size_t(i0 + r) * p.D + k0 + c] : 0.f;
      Bs[c][r] = (j0 + r < p.NB) ? Bm[size_t(j0 + r) * p.D + k0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kGK; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) { a[u] = As[c][ty * 4 + u]; b[u] = Bs[c][tx * 4 + u]; }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(a[u], b[w], acc[u][w]);
    }
    __syncthreads();
  }
  float* S = p.scores + size_t(bh) * p.NB * p.NB;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty * 4 + u;
    if (i >= p.NB) continue;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int j = j0 + tx * 4 + w;
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

__global__ void rowstats_kernel(SelectParams p, int warps, int stride) {
  extern __shared__ uint32_t sh_rs[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.y;
  const int i = blockIdx.x * warps + warp;
  if (i >= p.NB) return;
  const float* S = p.scores + (size_t(bh) * p.NB + i) * p.NB;
  float m = -INFINITY;
  for (int j = lane; j < p.NB; j += 32) m = fmaxf(m, S[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.f;
  for (int j = lane; j < p.NB; j += 32) l += expf(S[j] - m);
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
      if (keys[j] > kth) acc += expf(S[j] - m) / l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    sharp = acc + float(kk - n_gt) * (expf(order_key_to_float(kth) - m) / l);
  }
  if (lane == 0) {
    p.rowmax[size_t(bh) * p.NB + i] = m;
    p.rowsum[size_t(bh) * p.NB + i] = l;
    p.sharp[size_t(bh) * p.NB + i] = sharp;
  }
}

// ---------------------------------------------------------------------------
// out_c[bh, i, :] = sum_j P[i, j] * vmean[bh, j, :],  P = exp(s - m) / l.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) outc_kernel(SelectParams p) {
  __shared__ float Ps[kGK][kGT + 4];
  __shared__ float Vs[kGK][kGT + 4];
  __shared__ float sm[kGT], sl[kGT];
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kGT, d0 = blockIdx.x * kGT;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const float* S = p.scores + size_t(bh) * p.NB * p.NB;
  const float* V = p.vmean + size_t(bh) * p.NB * p.D;
  if (threadIdx.x < kGT) {
    const int i = i0 + threadIdx.x;
    sm[threadIdx.x] = (i < p.NB) ? p.rowmax[size_t(bh) * p.NB + i] : 0.f;
    sl[threadIdx.x] = (i < p.NB) ? p.rowsum[size_t(bh) * p.NB + i] : 1.f;
  }
  __syncthreads();
  float acc[4][4] = {};
  for (int j0 = 0; j0 < p.NB; j0 += kGK) {
    for (int e = threadIdx.x; e < kGT * kGK; e += 256) {
      const int r = e / kGK, c = e % kGK;
      const int i = i0 + r, j = j0 + c;
      Ps[c][r] = (i < p.NB && j < p.NB) ? expf(S[size_t(i) * p.NB + j] - sm[r]) / sl[r] : 0.f;
      const int jr = e / kGT, dc = e % kGT;
      Vs[jr][dc] = (j0 + jr < p.NB && d0 + dc < p.D) ? V[size_t(j0 + jr) * p.D + d0 + dc] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kGK; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) { a[u] = Ps[c][ty * 4 + u]; b[u] = Vs[c][tx * 4 + u]; }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(a[u], b[w], acc[u][w]);
    }
    __syncthreads();
  }
  float* O = p.outc + size_t(bh) * p.NB * p.D;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty * 4 + u;
    if (i >= p.NB) continue;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int d = d0 + tx * 4 + w;
      if (d < p.D) O[size_t(i) * p.D + d] = acc[u][w];
    }
  }
}

// ---------------------------------------------------------------------------
// colsum[bh, j] = sum over target rows i < n_t of P[i, n_t + j].  A CTA owns
// 32 columns; its 8 row groups each add every 8th row in increasing order and
// the 8 partial sums are combined in a fixed order (deterministic).
// ---------------------------------------------------------------------------
__global__ void colsum_kernel(SelectParams p) {
  __shared__ float part[8][33];
  const int bh = blockIdx.y;
  const int c = threadIdx.x, g = threadIdx.y;
  const int j = blockIdx.x * 32 + c;
  const float* M = p.rowmax + size_t(bh) * p.NB;
  const float* L = p.rowsum + size_t(bh) * p.NB;
  float acc = 0.f;
  if (j < p.n_s) {
    const float* S = p.scores + size_t(bh) * p.NB * p.NB + p.n_t + j;
    for (int i = g; i < p.n_t; i += 8) acc += expf(S[size_t(i) * p.NB] - M[i]) / L[i];
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

cudaError_t launch_compressed_attention(const SelectParams& p, cudaStream_t stream) {
  const int BH = p.B * p.H;
  dim3 g1((p.NB + kGT - 1) / kGT, (p.NB + kGT - 1) / kGT, BH);
  scores_kernel<<<g1, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const int stride = p.n_t > 0 ? p.n_t : 1;
  int warps = 8;
  auto rs_smem = [&](int w) { return size_t(w) * stride * sizeof(uint32_t) + size_t(w) * 256 * sizeof(uint32_t); };
  while (warps > 1 && rs_smem(warps) > 96 * 1024) warps >>= 1;
  const size_t smem = rs_smem(warps);
  if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(rowstats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  dim3 g2((p.NB + warps - 1) / warps, BH);
  rowstats_kernel<<<g2, warps * 32, smem, stream>>>(p, warps, stride);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  dim3 g3((p.D + kGT - 1) / kGT, (p.NB + kGT - 1) / kGT, BH);
  outc_kernel<<<g3, 256, 0, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  if (p.n_s > 0) {
    dim3 g4((p.n_s + 31) / 32, BH);
    colsum_kernel<<<g4, dim3(32, 8), 0, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace icsa
