// Stage 2 (continued): block selections and the extended-KV block table.
//
//  * in-context retrieval (editing_sparse_attention.py:126-136): the topK
//    source blocks with the largest column sums, in descending order;
//  * sharpness split (:162-172): all query blocks in descending sharpness;
//    the first num_flat go to dense attention, the rest to sparse attention;
//  * extended KV (:138-159): instead of materialising
//    new_k = [k[:t] | gathered source blocks], a table gives the first row of
//    every 64-row extended-KV block inside k (t_seq_len % 64 == 0), and the
//    block sums of the extended KV (tilelang reduce_kv_kernel) are gathered
//    from the stage-1 sums.  For t_seq_len % 64 != 0 the extended K/V are
//    materialised (blocks straddle the target/source seam) and pooled again;
//  * per-sparse-block top-k (tilelang_host.py:170-173): fp32
//    QC . KC^T against every extended-KV block, keep top_k.
#include "icsa_kernels.cuh"
#include "icsa_sort.cuh"

namespace icsa {

namespace {

// ---------------------------------------------------------------------------
// Sort one row of fp32 keys per CTA (descending, ties to the lower index) and
// write the first `keep` indices.
// ---------------------------------------------------------------------------
__global__ void sort_select_kernel(const float* keys, int n, int keep, int* out, int pow2) {
  extern __shared__ uint64_t sh_keys[];
  const int row = blockIdx.x;
  const float* k = keys + size_t(row) * n;
  for (int i = threadIdx.x; i < pow2; i += blockDim.x)
    sh_keys[i] = (i < n) ? select_key(k[i], uint32_t(i)) : 0ull;
  __syncthreads();
  bitonic_sort_desc(sh_keys, pow2, threadIdx.x, blockDim.x, BlockSync{});
  for (int i = threadIdx.x; i < keep; i += blockDim.x) out[size_t(row) * keep + i] = int(select_key_index(sh_keys[i]));
}

cudaError_t launch_sort_select(const float* keys, int rows, int n, int keep, int* out, cudaStream_t stream) {
  if (rows == 0 || keep == 0) return cudaSuccess;
  const int pow2 = next_pow2(n);
  const size_t smem = size_t(pow2) * sizeof(uint64_t);
  if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(sort_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  sort_select_kernel<<<rows, 512, smem, stream>>>(keys, n, keep, out, pow2);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Extended-KV block table.  aligned != 0: kv_rows points into k itself and
// kc/vc rows are gathered from the stage-1 block sums.  aligned == 0: kv_rows
// indexes the materialised buffer (block j starts at row 64 j) and only the
// padding rows of kc/vc are cleared here (the pool pass fills the rest).
// ---------------------------------------------------------------------------
__global__ void extended_kv_kernel(SelectParams p, int aligned) {
  const int bh = blockIdx.y;
  const int j = blockIdx.x;  // extended-KV block, 0 .. nkv_pad-1
  const size_t dst = (size_t(bh) * p.nkv_pad + j) * p.D;
  int src_block = -1;
  if (j < p.nkv) {
    if (aligned) {
      src_block = (j < p.n_t) ? j : p.n_t + p.sel[size_t(bh) * p.topK + (j - p.n_t)];
      if (threadIdx.x == 0) p.kv_rows[size_t(bh) * p.nkv + j] = src_block * kBlock;
    } else {
      if (threadIdx.x == 0) p.kv_rows[size_t(bh) * p.nkv + j] = j * kBlock;
      return;
    }
  }
  const size_t src = (size_t(bh) * p.NB + (src_block < 0 ? 0 : src_block)) * p.D;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    const __nv_bfloat16 z = __float2bfloat16(0.f);
    p.kc[dst + d] = src_block < 0 ? z : p.ksum[src + d];
    p.vc[dst + d] = src_block < 0 ? z : p.vsum[src + d];
  }
}

// ---------------------------------------------------------------------------
// Materialise the extended K/V (t_seq_len % 64 != 0) as bf16 [B, nkv*64, H, D]:
// rows < t copy k[:t]; rows t .. tkv-1 copy the selected source blocks from
// the zero-padded k starting at row (t // 64) * 64 (the reference's gather
// offset, :148-152); rows >= tkv are zero (the tilelang host pads them).
// ---------------------------------------------------------------------------
__global__ void gather_extended_kernel(SelectParams p) {
  const int r = blockIdx.x;  // extended row
  const int b = blockIdx.y;
  const int HD = p.H * p.D;
  const int rows_ext = p.nkv * kBlock;
  for (int c = threadIdx.x * 8; c < HD; c += blockDim.x * 8) {
    const int h = c / p.D;
    long src_row = -1;
    if (r < p.t_seq_len) {
      src_row = r;
    } else if (r < p.tkv) {
      const int q = (r - p.t_seq_len) / kBlock, o = (r - p.t_seq_len) % kBlock;
      const int blk = p.sel[(size_t(b) * p.H + h) * p.topK + q];
      src_row = long(p.n_t) * kBlock + long(blk) * kBlock + o;
      if (src_row >= p.S) src_row = -1;
    }
    uint4 kz = make_uint4(0, 0, 0, 0), vz = kz;
    if (src_row >= 0) {
      const size_t s = (size_t(b) * p.S + src_row) * HD + c;
      kz = *reinterpret_cast<const uint4*>(p.k_src + s);
      vz = *reinterpret_cast<const uint4*>(p.v_src + s);
    }
    const size_t d = (size_t(b) * rows_ext + r) * HD + c;
    *reinterpret_cast<uint4*>(p.newk + d) = kz;
    *reinterpret_cast<uint4*>(p.newv + d) = vz;
  }
}

// ---------------------------------------------------------------------------
// Per sparse query block: fp32 scores QC . KC^T against every extended-KV
// block (tilelang_host.py:172), then the top_k blocks (:173) by a warp radix
// select; ties go to the lower block index, and the selected set is written
// in increasing block order together with its bit set.
//
// CTA: `rows` (<= 8) sparse query blocks of one (b,h), 256 threads.  Scoring:
// thread <-> extended-KV block, 8 query rows register-blocked, the query sums
// transposed in shared memory ([D][8]) so each k value feeds 8 FMAs.
// Selection: warp w <-> query block w.
// ---------------------------------------------------------------------------
constexpr int kTopkThreads = 256;
constexpr int kTopkRowsMax = 8;

__global__ void __launch_bounds__(kTopkThreads) sparse_topk_kernel(SelectParams p, int rows) {
  extern __shared__ __align__(16) unsigned char sh_raw[];
  const int D = p.D, nkv = p.nkv;
  float* qT = reinterpret_cast<float*>(sh_raw);                                  // [D][8]
  uint32_t* keys = reinterpret_cast<uint32_t*>(qT + D * kTopkRowsMax);           // [rows][nkv]
  uint32_t* hist = keys + size_t(rows) * nkv;                                    // [8][256]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int r0 = blockIdx.x * rows;
  const int* order = p.order + size_t(bh) * p.NB + p.num_flat;
  for (int e = tid; e < kTopkRowsMax * D; e += kTopkThreads) {
    const int r = e / D, d = e % D;
    float v = 0.f;
    if (r < rows && r0 + r < p.n_sparse)
      v = __bfloat162float(p.qsum[(size_t(bh) * p.NB + order[r0 + r]) * D + d]);
    qT[d * kTopkRowsMax + r] = v;
  }
  __syncthreads();
  const __nv_bfloat16* KC = p.kc + size_t(bh) * p.nkv_pad * D;
  for (int col = tid; col < nkv; col += kTopkThreads) {
    float acc[kTopkRowsMax];
#pragma unroll
    for (int r = 0; r < kTopkRowsMax; ++r) acc[r] = 0.f;
    const __nv_bfloat16* kr = KC + size_t(col) * D;
    for (int d0 = 0; d0 < D; d0 += 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(kr + d0));
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
      float kf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(hv[i]);
        kf[2 * i] = f.x;
        kf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float4 a = reinterpret_cast<const float4*>(qT)[(d0 + e) * 2];
        const float4 b = reinterpret_cast<const float4*>(qT)[(d0 + e) * 2 + 1];
        acc[0] = fmaf(a.x, kf[e], acc[0]);
        acc[1] = fmaf(a.y, kf[e], acc[1]);
        acc[2] = fmaf(a.z, kf[e], acc[2]);
        acc[3] = fmaf(a.w, kf[e], acc[3]);
        acc[4] = fmaf(b.x, kf[e], acc[4]);
        acc[5] = fmaf(b.y, kf[e], acc[5]);
        acc[6] = fmaf(b.z, kf[e], acc[6]);
        acc[7] = fmaf(b.w, kf[e], acc[7]);
      }
    }
#pragma unroll
    for (int r = 0; r < kTopkRowsMax; ++r) {
      if (r < rows) {
        keys[size_t(r) * nkv + col] = float_order_key(acc[r]);
        if (p.blockscore != nullptr && r0 + r < p.n_sparse)
          p.blockscore[(size_t(bh) * p.n_sparse + r0 + r) * nkv + col] = acc[r];
      }
    }
  }
  __syncthreads();
  if (warp >= rows || r0 + warp >= p.n_sparse) return;
  const int r = r0 + warp;
  const uint32_t* myk = keys + size_t(warp) * nkv;
  int n_gt = 0;
  const uint32_t kth = warp_kth_largest(myk, nkv, p.top_k, hist + warp * 256, &n_gt);
  const int need_eq = p.top_k - n_gt;
  int* idx = p.sparse_idx + (size_t(bh) * p.n_sparse + r) * p.top_k;
  uint32_t* mask = p.sel_mask + (size_t(bh) * p.n_sparse + r) * (p.nkv_pad / 32);
  const uint32_t lt = (1u << lane) - 1u;
  int written = 0, eq_seen = 0;
  for (int c0 = 0; c0 < p.nkv_pad; c0 += 32) {
    const int col = c0 + lane;
    const uint32_t u = col < nkv ? myk[col] : 0u;
    const bool gt = col < nkv && u > kth;
    const bool eq = col < nkv && u == kth;
    const uint32_t eqm = __ballot_sync(0xffffffffu, eq);
    const bool take = gt || (eq && eq_seen + __popc(eqm & lt) < need_eq);
    const uint32_t selm = __ballot_sync(0xffffffffu, take);
    if (take) idx[written + __popc(selm & lt)] = col;
    if (lane == 0) mask[c0 / 32] = selm;
    written += __popc(selm);
    eq_seen += __popc(eqm);
  }
}

}  // namespace

cudaError_t launch_selection(const SelectParams& p, cudaStream_t stream) {
  const int BH = p.B * p.H;
  cudaError_t e = launch_sort_select(p.colsum, BH, p.n_s, p.topK, p.sel, stream);
  if (e != cudaSuccess) return e;
  return launch_sort_select(p.sharp, BH, p.NB, p.NB, p.order, stream);
}

cudaError_t launch_extended_kv(const SelectParams& p, cudaStream_t stream) {
  const int BH = p.B * p.H;
  const int aligned = (p.t_seq_len % kBlock) == 0;
  if (!aligned) {
    dim3 g(p.nkv * kBlock, p.B);
    gather_extended_kernel<<<g, 256, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  dim3 g(p.nkv_pad, BH);
  extended_kv_kernel<<<g, 128, 0, stream>>>(p, aligned);
  return cudaGetLastError();
}

cudaError_t launch_sparse_topk(const SelectParams& p, cudaStream_t stream) {
  if (p.n_sparse == 0) return cudaSuccess;
  const int BH = p.B * p.H;
  auto smem_for = [&](int rows) {
    return size_t(kTopkRowsMax) * p.D * sizeof(float) + size_t(rows) * p.nkv * sizeof(uint32_t) +
           size_t(kTopkRowsMax) * 256 * sizeof(uint32_t);
  };
  int rows = kTopkRowsMax;
  while (rows > 1 && smem_for(rows) > 200 * 1024) --rows;
  const size_t smem = smem_for(rows);
  if (smem > 220 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(sparse_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 g((p.n_sparse + rows - 1) / rows, BH);
  sparse_topk_kernel<<<g, kTopkThreads, smem, stream>>>(p, rows);
  return cudaGetLastError();
}

}  // namespace icsa
