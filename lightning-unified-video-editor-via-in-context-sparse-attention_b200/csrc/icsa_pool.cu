// Stage 1: 64-token block pooling of Q, K and V in one HBM pass.
//
// Reference behaviour restated here:
//   * editing level (editing_sparse_attention.py:37-55, :107-111): per block
//     mean = sum / block_size computed in the input dtype's arithmetic and
//     rounded back to the input dtype (the last block may be partial);
//   * sparse level (tilelang_kernels.py:33-120, reduce_q_kernel /
//     reduce_kv_kernel): per block SUM of the bf16-cast rows, accumulated in
//     fp32 and rounded to bf16.
// For bf16 inputs both come from one fp32 sum (mean = bf16(bf16(sum) / size));
// for fp32 inputs the bf16-rounded rows are summed separately, and the bf16
// copy that the tensor-core stages read is written in the same pass.
//
// Layout: input rows are [B, S, H*D] (row stride H*D); every thread owns 8
// consecutive features of a row (16-byte bf16 loads) and walks the 64 rows of
// one block, so a warp reads 512 contiguous bytes per row.  Outputs are
// head-major [B*H, block_stride, D].
#include "icsa_kernels.cuh"

namespace icsa {

namespace {

constexpr int kPoolThreads = 128;

template <typename T>
struct Vec8;

template <>
struct Vec8<__nv_bfloat16> {
  static ICSA_DEV void load(const __nv_bfloat16* p, float (&f)[8]) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};

template <>
struct Vec8<float> {
  static ICSA_DEV void load(const float* p, float (&f)[8]) {
    float4 a = __ldg(reinterpret_cast<const float4*>(p));
    float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

ICSA_DEV void store_bf16x8(__nv_bfloat16* dst, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(dst) = u;
}

ICSA_DEV void store_f32x8(float* dst, const float (&f)[8]) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

template <typename T>
ICSA_DEV void pool_block(const PoolParams& p, const PoolTensor& t, int b, int nb) {
  const int HD = p.H * p.D;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= HD) return;
  const int row0 = nb * kBlock;
  const int rows = min(kBlock, p.S - row0);
  const T* src = reinterpret_cast<const T*>(t.x) + (size_t(b) * p.S + row0) * HD + col;

  float sum[8], sum_bf[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { sum[i] = 0.f; sum_bf[i] = 0.f; }

  constexpr bool kF32 = sizeof(T) == 4;
  __nv_bfloat16* copy = (kF32 && t.copy_bf16 != nullptr)
                            ? t.copy_bf16 + (size_t(b) * p.S + row0) * HD + col
                            : nullptr;

  int r = 0;
  // Unrolled main loop keeps 8 independent 16/32-byte loads in flight.
  for (; r + 8 <= rows; r += 8) {
    float f[8][8];
#pragma unroll
    for (int u = 0; u < 8; ++u) Vec8<T>::load(src + size_t(r + u) * HD, f[u]);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sum[i] += f[u][i];
        if (kF32) sum_bf[i] += bf16_round(f[u][i]);
      }
      if (kF32 && copy != nullptr) store_bf16x8(copy + size_t(r + u) * HD, f[u]);
    }
  }
  for (; r < rows; ++r) {
    float f[8];
    Vec8<T>::load(src + size_t(r) * HD, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sum[i] += f[i];
      if (kF32) sum_bf[i] += bf16_round(f[i]);
    }
    if (kF32 && copy != nullptr) store_bf16x8(copy + size_t(r) * HD, f);
  }

  const int h = col / p.D;
  const int d = col % p.D;
  const size_t o = ((size_t(b) * p.H + h) * p.block_stride + nb) * p.D + d;
  float sb[8], mean[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (kF32) {
      sb[i] = sum_bf[i];
      mean[i] = sum[i] / float(rows);
      if (t.round_mean_bf16) mean[i] = bf16_round(mean[i]);
    } else {
      sb[i] = sum[i];
      // bf16 arithmetic of the reference: bf16(sum) / size, rounded to bf16.
      mean[i] = bf16_round(bf16_round(sum[i]) / float(rows));
    }
  }
  if (t.sum_bf16 != nullptr) store_bf16x8(t.sum_bf16 + o, sb);
  if (t.mean_f32 != nullptr) store_f32x8(t.mean_f32 + o, mean);
}

__global__ void __launch_bounds__(kPoolThreads) pool_kernel(PoolParams p) {
  const int which = blockIdx.z % 3;  // 0: q, 1: k, 2: v
  const int b = blockIdx.z / 3;
  const PoolTensor& t = p.t[which];
  if (t.x == nullptr) return;
  if (t.dtype == ICSA_F32)
    pool_block<float>(p, t, b, blockIdx.y);
  else
    pool_block<__nv_bfloat16>(p, t, b, blockIdx.y);
}

}  // namespace

cudaError_t launch_pool(const PoolParams& p, cudaStream_t stream) {
  const int HD = p.H * p.D;
  const int vec_lanes = HD / 8;
  // a row of few heads is narrower than 128 lanes: size the CTA to it (whole
  // warps) so that more CTAs, and more loads, fit on an SM
  const int threads = vec_lanes < kPoolThreads ? (vec_lanes + 31) / 32 * 32 : kPoolThreads;
  dim3 grid((vec_lanes + threads - 1) / threads, p.num_blocks, 3 * p.B);
  pool_kernel<<<grid, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace icsa
