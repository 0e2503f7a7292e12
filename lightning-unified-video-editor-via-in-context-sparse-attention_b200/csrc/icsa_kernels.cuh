// Parameter blocks and launchers of the three stages (pool, select, attend).
#pragma once

#include "icsa_common.cuh"

// Sets the message returned by icsa_last_error() on the calling thread
// (library-internal, defined in icsa_capi.cu).
extern "C" void icsa_set_last_error(const char* msg);

namespace icsa {

// ---------------------------------------------------------------- stage 1 --
struct PoolTensor {
  const void* x;             // [B, S, H, D] input rows (nullptr: skip this tensor)
  int dtype;                 // ICSA_BF16 / ICSA_F32
  __nv_bfloat16* sum_bf16;   // [B*H, block_stride, D] bf16 block sums (may be nullptr)
  float* mean_f32;           // [B*H, block_stride, D] block means (may be nullptr)
  __nv_bfloat16* copy_bf16;  // [B, S, H, D] bf16 copy of an f32 input (may be nullptr)
  int round_mean_bf16;       // f32 input whose compressed attention runs in bf16 (autocast)
};

struct PoolParams {
  int B, S, H, D;
  int num_blocks;    // ceil(S / 64)
  int block_stride;  // block count of the output layout (>= num_blocks)
  PoolTensor t[3];
};

cudaError_t launch_pool(const PoolParams& p, cudaStream_t stream);

// ---------------------------------------------------------------- stage 2 --
struct SelectParams {
  int B, H, D, S;
  int NB, n_t, n_s, topK, num_flat, n_sparse, k_sparsity, top_k;
  int nkv, nkv_pad, tkv, t_seq_len;
  float inv_sqrt_d_div;  // divisor sqrt(D) of the reference (QK /= sqrt(D))
  // stage-1 outputs
  const float* qmean;
  const float* kmean;
  const float* vmean;
  const __nv_bfloat16* qsum;
  const __nv_bfloat16* ksum;
  const __nv_bfloat16* vsum;
  // stage-2 outputs
  float* scores;   // [BH, NB, NB]
  float* rowmax;   // [BH, NB]
  float* rowsum;   // [BH, NB]
  float* sharp;    // [BH, NB]
  float* colsum;   // [BH, n_s]
  float* outc;     // [BH, NB, D]
  int* sel;        // [BH, topK]
  int* order;      // [BH, NB]
  int* kv_rows;    // [BH, nkv]
  __nv_bfloat16* kc;  // [BH, nkv_pad, D]
  __nv_bfloat16* vc;  // [BH, nkv_pad, D]
  int* sparse_idx;    // [BH, n_sparse, top_k]
  uint32_t* sel_mask; // [BH, n_sparse, nkv_pad / 32]
  float* blockscore;  // [BH, n_sparse, nkv] per-sparse-block scores
  // unaligned t_seq_len: materialised extended KV
  const __nv_bfloat16* k_src;  // bf16 [B, S, H, D] source of the gather
  const __nv_bfloat16* v_src;
  __nv_bfloat16* newk;         // [B, nkv*64, H, D]
  __nv_bfloat16* newv;
  int means_bf16;              // qmean and kmean hold bf16 values (tensor-core scores)
  int vmean_bf16;              // vmean holds bf16 values (tensor-core out_c)
  int* err;                    // workspace status word (bounded waits)
};

// Compressed attention: scores, row statistics and in-context column sums on
// `stream`; out_compress (which only the attention epilogue reads) on
// `outc_stream`, which the caller orders after the row statistics.
cudaError_t launch_compressed_scores(const SelectParams& p, cudaStream_t stream);
// The scores alone on tcgen05 (means_bf16 and D = 64 or 128).
cudaError_t launch_scores_tc(const SelectParams& p, cudaStream_t stream);
// out_c on tcgen05 (vmean_bf16 and D = 64 or 128; part of launch_outc).
cudaError_t launch_outc_tc(const SelectParams& p, cudaStream_t stream);
// blockscore = QC[sparse blocks] . KC^T on tcgen05 (part of launch_sparse_topk).
cudaError_t launch_blockscore_tc(const SelectParams& p, cudaStream_t stream);
cudaError_t launch_outc(const SelectParams& p, cudaStream_t stream);
cudaError_t launch_colsum(const SelectParams& p, cudaStream_t stream);
cudaError_t launch_selection(const SelectParams& p, cudaStream_t stream);
cudaError_t launch_extended_kv(const SelectParams& p, cudaStream_t stream);
cudaError_t launch_sparse_topk(const SelectParams& p, cudaStream_t stream);

// ---------------------------------------------------------------- stage 3 --
struct AttnParams {
  int B, S, H, NB;
  int num_flat, n_sparse;        // query blocks per (b, h)
  int flat_tiles, sparse_tiles;  // tiles per (b, h) = ceil(count / 2)
  int nkv, nkv_pad, tkv, top_k;
  float scale_log2;              // log2(e) / sqrt(D)
  const int* order;              // [BH, NB]: flat blocks first, then sparse
  const int* kv_rows;            // [BH, nkv]
  const int* sparse_idx;         // [BH, n_sparse, top_k]
  const uint32_t* sel_mask;      // [BH, n_sparse, nkv_pad/32]
  const float* outc;             // [BH, NB, D]
  int outc_bf16;
  // alpha
  int alpha_mode, alpha_dtype, ca_bf16;
  float alpha_scalar;
  const void* alpha;
  long long alpha_strides[4];
  // output [B, S, H, D]
  void* out;
  int out_dtype;
  int out_tma;                   // 1: bf16 output written by TMA stores through maps.o
  int* err;
};

struct AttnMaps {
  CUtensorMap q;   // bf16 [B, S, H, D]     box {64, 1, 64, 1}
  CUtensorMap k;   // bf16 [B, Skv, H, D]   box {64, 1, 64, 1}
  CUtensorMap v;
  CUtensorMap kc;  // bf16 [BH, nkv_pad, D] box {64, 128, 1}
  CUtensorMap vc;
  CUtensorMap o;   // bf16 output [B, S, H, D] box {64, 1, 64, 1} (when out_tma)
};

// Dense tiles of the flat query blocks, two 128-row tiles per CTA.
cudaError_t launch_flat_attention(const AttnParams& p, const AttnMaps& maps, int D, cudaStream_t stream);
// Dense tiles of the flat query blocks for D = 128 on SM pairs (cta_group::2).
cudaError_t launch_dense_pair_attention(const AttnParams& p, const AttnMaps& maps, cudaStream_t stream);
// Block-sparse tiles (exact top_k blocks + interval term), P kept in TMEM.
cudaError_t launch_sparse_attention(const AttnParams& p, const AttnMaps& maps, int D, cudaStream_t stream);

// ------------------------------------------------- DiT output projections --
// x[r, c] += bf16(a[r, :] . w[c, :] + bias[c]) * gate[r / rows_per_batch, c]
// (gate nullptr: + bf16(...)); a_map / w_map: bf16 [M, K] / [N, K] with
// {64, 128} boxes and 128-byte swizzle.
cudaError_t launch_linear_residual(int M, int N, int K, const CUtensorMap& a_map, const CUtensorMap& w_map,
                                   const __nv_bfloat16* bias, float* x, int64_t ldx, const float* gate,
                                   int64_t gate_bs, int rows_per_batch, int num_sms, cudaStream_t stream);

// Device addresses of the per-device sticky status words of the translation
// units whose kernels have bounded waits (see report_error).
cudaError_t sticky_status_dense_pair(int** out);
cudaError_t sticky_status_flat(int** out);
cudaError_t sticky_status_sparse(int** out);
cudaError_t sticky_status_selftest(int** out);
cudaError_t sticky_status_gemm(int** out);
cudaError_t sticky_status_scores(int** out);

}  // namespace icsa
