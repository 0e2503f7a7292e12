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
// Per sparse query block: scores against all extended-KV block sums and the
// top_k selection.  One warp per query block, `warps` blocks of one (b,h)
// per CTA; KC is staged through shared memory 64 rows at a time.
// ---------------------------------------------------------------------------
constexpr int kKcChunk = 64;

__global__ void sparse_topk_kernel(SelectParams p, int warps, int pow2) {
  extern __shared__ __align__(16) unsigned char sh_raw[];
  const int D = p.D;
  uint64_t* keys = reinterpret_cast<uint64_t*>(sh_raw);                  // [warps][pow2]
  float* qrow = reinterpret_cast<float*>(keys + size_t(warps) * pow2);  // [warps][D]
  float* kct = qrow + size_t(warps) * D;                                 // [64][D+1]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.y;
  const int r = blockIdx.x * warps + warp;  // sparse query block rank
  const bool active = r < p.n_sparse;
  if (active) {
    const int blk = p.order[size_t(bh) * p.NB + p.num_flat + r];
    const __nv_bfloat16* qs = p.qsum + (size_t(bh) * p.NB + blk) * D;
    for (int d = lane; d < D; d += 32) qrow[warp * D + d] = __bfloat162float(qs[d]);
  }
  uint64_t* mykeys = keys + size_t(warp) * pow2;
  for (int j = lane; j < pow2; j += 32) mykeys[j] = 0ull;
  const __nv_bfloat16* KC = p.kc + size_t(bh) * p.nkv_pad * D;
  for (int c0 = 0; c0 < p.nkv; c0 += kKcChunk) {
    __syncthreads();
    for (int e = threadIdx.x; e < kKcChunk * D; e += blockDim.x) {
      const int rr = e / D, d = e % D;
      kct[rr * (D + 1) + d] = (c0 + rr < p.nkv) ? __bfloat162float(KC[size_t(c0 + rr) * D + d]) : 0.f;
    }
    __syncthreads();
    if (active) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int cc = lane + 32 * half;
        const int col = c0 + cc;
        if (col < p.nkv) {
          float acc = 0.f;
          const float* kr = kct + cc * (D + 1);
          const float* qr = qrow + warp * D;
          for (int d = 0; d < D; ++d) acc = fmaf(qr[d], kr[d], acc);
          mykeys[col] = select_key(acc, uint32_t(col));
          if (p.blockscore != nullptr) p.blockscore[(size_t(bh) * p.n_sparse + r) * p.nkv + col] = acc;
        }
      }
    }
  }
  __syncwarp();
  if (!active) return;
  bitonic_sort_desc(mykeys, pow2, lane, 32, WarpSync{});
  int* idx = p.sparse_idx + (size_t(bh) * p.n_sparse + r) * p.top_k;
  for (int i = lane; i < p.top_k; i += 32) idx[i] = int(select_key_index(mykeys[i]));
  // bit set of the selected blocks, one 32-bit word per lane step
  const int words = p.nkv_pad / 32;
  uint32_t* mask = p.sel_mask + (size_t(bh) * p.n_sparse + r) * words;
  for (int w = lane; w < words; w += 32) {
    uint32_t bits = 0;
    for (int i = 0; i < p.top_k; ++i) {
      const uint32_t sel = select_key_index(mykeys[i]);
      if (sel / 32 == uint32_t(w)) bits |= 1u << (sel % 32);
    }
    mask[w] = bits;
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
  const int pow2 = next_pow2(p.nkv);
  int warps = 8;
  auto smem_for = [&](int w) {
    return size_t(w) * pow2 * sizeof(uint64_t) + size_t(w) * p.D * sizeof(float) +
           size_t(kKcChunk) * (p.D + 1) * sizeof(float);
  };
  while (warps > 1 && smem_for(warps) > 160 * 1024) warps >>= 1;
  const size_t smem = smem_for(warps);
  if (smem > 220 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(sparse_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 g((p.n_sparse + warps - 1) / warps, BH);
  sparse_topk_kernel<<<g, warps * 32, smem, stream>>>(p, warps, pow2);
  return cudaGetLastError();
}

}  // namespace icsa
