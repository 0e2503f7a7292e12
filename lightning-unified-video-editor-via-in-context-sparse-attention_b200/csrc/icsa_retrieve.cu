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
//    QC . KC^T against every extended-KV block (a tensor-core block GEMM),
//    keep top_k.
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
  wait_prior_grid();
  for (int i = threadIdx.x; i < pow2; i += blockDim.x)
    sh_keys[i] = (i < n) ? select_key(k[i], uint32_t(i)) : 0ull;
  __syncthreads();
  bitonic_sort_desc(sh_keys, pow2, threadIdx.x, blockDim.x);
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
  const int threads = pow2 < 1024 ? pow2 : 1024;  // one key per thread up to 1024 keys
  return launch_chained(sort_select_kernel, dim3(rows), dim3(threads), smem, stream, keys, n, keep, out, pow2);
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
  wait_prior_grid();
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
  wait_prior_grid();
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
// Per sparse query block: the top_k extended-KV blocks (tilelang_host.py:173)
// of its fp32 scores QC . KC^T (:172, computed on the tensor cores into
// p.blockscore beforehand), by a warp radix select; ties go to the lower block
// index, and the selected set is written in increasing block order together
// with its bit set.
//
// CTA: `rows` (<= 8) sparse query blocks of one (b,h), warp w <-> query
// block w; the CTA first stages the rows' order-preserving keys in shared
// memory.
// ---------------------------------------------------------------------------
constexpr int kTopkThreads = 256;
constexpr int kTopkRowsMax = 8;

__global__ void __launch_bounds__(kTopkThreads) sparse_topk_kernel(SelectParams p, int rows) {
  extern __shared__ __align__(16) unsigned char sh_raw[];
  const int nkv = p.nkv;
  uint32_t* keys = reinterpret_cast<uint32_t*>(sh_raw);  // [rows][nkv]
  uint32_t* hist = keys + size_t(rows) * nkv;             // [8][256]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int r0 = blockIdx.x * rows;
  const int valid = min(rows, p.n_sparse - r0);
  const float* bs = p.blockscore + (size_t(bh) * p.n_sparse + r0) * nkv;
  wait_prior_grid();
  for (int e = tid; e < valid * nkv; e += kTopkThreads) keys[e] = float_order_key(bs[e]);
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
    cudaError_t e = launch_chained(gather_extended_kernel, g, dim3(256), 0, stream, p);
    if (e != cudaSuccess) return e;
  }
  dim3 g(p.nkv_pad, BH);
  return launch_chained(extended_kv_kernel, g, dim3(128), 0, stream, p, aligned);
}

cudaError_t launch_sparse_topk(const SelectParams& p, cudaStream_t stream) {
  if (p.n_sparse == 0) return cudaSuccess;
  const int BH = p.B * p.H;
  cudaError_t e = launch_blockscore_tc(p, stream);
  if (e != cudaSuccess) return e;
  auto smem_for = [&](int rows) {
    return size_t(rows) * p.nkv * sizeof(uint32_t) + size_t(kTopkRowsMax) * 256 * sizeof(uint32_t);
  };
  int rows = kTopkRowsMax;
  while (rows > 1 && smem_for(rows) > 200 * 1024) --rows;
  const size_t smem = smem_for(rows);
  if (smem > 220 * 1024) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(sparse_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 g((p.n_sparse + rows - 1) / rows, BH);
  return launch_chained(sparse_topk_kernel, g, dim3(kTopkThreads), smem, stream, p, rows);
}

}  // namespace icsa
