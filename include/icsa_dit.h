/*
 * icsa_dit.h -- C ABI of the fused elementwise stages of one Wan 2.2 DiT
 * block (libicsa.so), the code that surrounds the in-context sparse
 * attention call in the reference's model (model.py:128-288).
 *
 * The GEMMs of the block (q/k/v/o projections, cross-attention projections,
 * FFN) are plain library GEMMs and stay with the caller; these entry points
 * are the memory-bound passes between them, each one HBM pass:
 *
 *   icsa_dit_modulated_norm  LayerNorm, then `* scale + shift`, written as
 *                            the bf16 operand of the next GEMM
 *                            (model.py:256 `norm1(x).float() * (1 + e[1]) + e[0]`,
 *                             :263 `norm2(x).float() * (1 + e[4]) + e[3]`,
 *                             :262 `norm3(x)` with its affine weight / bias,
 *                             :288 the head's norm; WanLayerNorm :116-121)
 *   icsa_dit_norm_rope       RMSNorm of q and k over the model width, the 3D
 *                            rotary embedding in float64, v passed through,
 *                            all written straight into the layout the
 *                            attention (or the Ulysses all-to-all) reads, and
 *                            the per-token gate alpha_1
 *                            (model.py:152-170, rope_apply :69-95, WanRMSNorm :102-113)
 *   icsa_dit_gated_residual  x += y * gate in float32
 *                            (model.py:259 `x + y * e[2]`, :262 `x + cross_attn(..)`,
 *                             :265 `x + y * e[5]`)
 *
 * Conventions as in icsa.h: plain device pointers, element counts and
 * strides in elements, asynchronous on `stream`, an icsa_status return and
 * icsa_last_error() for the message.  bf16 buffers must be 16-byte aligned
 * and their leading dimensions multiples of 8 elements.
 */
#ifndef ICSA_DIT_H_
#define ICSA_DIT_H_

#include "icsa.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * out[r, c] = bf16( n[r, c] * scale[b, c] + shift[b, c] ),  b = r / rows_per_batch,
 * n = LayerNorm(x[r, :]) without affine terms (biased variance, eps inside the
 * square root), rounded to bf16 first when `round_norm_bf16` is set (the
 * reference's `type_as(x)` for a bf16 residual stream).  The product and the
 * sum are rounded separately, as the reference's two float32 ops are.
 *   x:     [rows, ldx] of x_dtype (ICSA_F32 or ICSA_BF16), C columns used
 *   scale, shift: float32, row b at b * batch_stride (0 = one row for all)
 *   out:   bf16 [rows, C], contiguous
 * C must be a multiple of 8 and at most 8192.
 */
ICSA_API int icsa_dit_modulated_norm(const void* x, int x_dtype, int64_t ldx, int rows, int C, int rows_per_batch,
                                     const float* scale, int64_t scale_batch_stride, const float* shift,
                                     int64_t shift_batch_stride, float eps, int round_norm_bf16, void* out,
                                     cudaStream_t stream);

/*
 * Up to three vectors of width C = heads * D per row, taken from bf16 rows of
 * leading dimension `ld` (for a fused q|k|v GEMM output, src[j] = base + j*C).
 * Vector j gets, when norm_weight[j] is non-NULL, the reference's WanRMSNorm:
 *     bf16( bf16( x * rsqrt(mean(x^2) + eps) ) * weight )
 * then, when rope[j] is set, the rotary embedding of rope_apply computed in
 * float64: pair i of head h of token t is multiplied by (cos, sin) =
 * rope_table[pos][i], pos being the token's frame, row or column index for
 * pairs [0, split1), [split1, split2), [split2, D/2); tokens whose
 * token_pos[t].rotate is 0 pass unrotated (the reference's padding with ones).
 * The result is stored as dst_dtype[j] at element offset
 *     b*dst_batch_stride + (h / heads_per_group)*dst_group_stride
 *       + t_local*dst_token_stride + (h % heads_per_group)*D + d
 * so that [B, S, H, D] (one group) and the per-destination blocks of an
 * all-to-all are both plain layouts.
 * The optional gate reads column `gate_src` of every row (bf16, same ld) and
 * writes the reference's alpha_1 = (sigmoid(a) - 0.5) * 0.5 with each op
 * rounded to bf16 (model.py:162), to gate_dst[r] (bf16 [rows]).
 */
typedef struct icsa_dit_norm_rope_desc {
  int rows, C, D;
  int64_t ld;
  int rows_per_batch;       /* tokens of one batch element in this call (t_local < rows_per_batch) */
  int token_offset;         /* global token index of t_local = 0                         */
  float eps;
  int count;                /* vectors per row, 1..3                                     */
  const void* src[3];
  const void* norm_weight[3];
  int rope[3];
  void* dst[3];
  int dst_dtype[3];
  int heads_per_group;
  int64_t dst_batch_stride, dst_group_stride, dst_token_stride;
  const double* rope_table; /* [rope_positions][D/2][2] (cos, sin)                       */
  int rope_positions;
  const int* token_pos;     /* [global tokens][4]: frame, row, column, rotate             */
  int token_count;          /* entries of token_pos                                      */
  int rope_split1, rope_split2;
  const void* gate_src;     /* NULL: no gate                                              */
  void* gate_dst;
} icsa_dit_norm_rope_desc;

ICSA_API int icsa_dit_norm_rope(const icsa_dit_norm_rope_desc* desc, cudaStream_t stream);

/*
 * The same pass with the attention's block pooling done on the producer side
 * (the first step of the reference's call, editing_sparse_attention.py:37-55
 * and :107-111, `compress_seq` of the float32 rotary output): every vector is
 * written as bf16 (dst_dtype must be ICSA_BF16), and for each vector j with
 * mean[j] set, the float32 mean of every 64-token block is written too:
 * rows summed in order and divided by 64, rounded to bf16 values when
 * round_mean_bf16 is set (the compressed attention then runs in bf16), i.e.
 * bit for bit what icsa_pool computes from the float32 vector.  Mean of
 * block k of head h, batch b:
 *     b*mean_batch_stride + (h / heads_per_group)*mean_group_stride
 *       + ((h % heads_per_group)*(rows_per_batch/64) + k)*D + d
 * rows_per_batch must be a multiple of 64.  rs_scratch: float workspace of
 * count * rows entries (the per-row RMSNorm factors).
 * Optionally, with sum[j] set, the bf16 sum of every block of the written
 * bf16 values (rows summed in order in float32, rounded once: what icsa_pool
 * writes as the block sums), at the same offsets; and with bf16_mean[j] set,
 * mean[j] is instead the bf16-arithmetic mean bf16(bf16(sum) / 64) of the
 * written bf16 values, what icsa_pool computes for a bf16 vector.
 * A sequence-parallel caller exchanges bf16 vectors and these block
 * statistics instead of float32 vectors, and hands them to the attention in
 * place of its pooling stage (q and k: float32 means and bf16 sums; v: bf16
 * means and sums).
 */
typedef struct icsa_dit_norm_rope_pool_desc {
  icsa_dit_norm_rope_desc base;
  void* mean[3];
  int64_t mean_batch_stride, mean_group_stride;
  int round_mean_bf16;
  float* rs_scratch;
  void* sum[3];          /* bf16 block sums, or NULL */
  int bf16_mean[3];      /* 1: mean[j] in the bf16 arithmetic of a bf16 vector */
} icsa_dit_norm_rope_pool_desc;

ICSA_API int icsa_dit_norm_rope_pool(const icsa_dit_norm_rope_pool_desc* desc, cudaStream_t stream);

/*
 * x[r, c] = x[r, c] + y[r, c] * gate[b, c]  in float32 (product and sum
 * rounded separately), b = r / rows_per_batch; gate NULL means x + y.
 *   x: float32 [rows, C] contiguous;  y: bf16 [rows, ldy];  gate: float32,
 *   row b at b * gate_batch_stride.
 */
ICSA_API int icsa_dit_gated_residual(float* x, const void* y, int64_t ldy, int rows, int C, int rows_per_batch,
                                     const float* gate, int64_t gate_batch_stride, cudaStream_t stream);

/*
 * A linear layer with the residual update fused into its epilogue:
 *     x[r, c] = x[r, c] + bf16( a[r, :] . w[c, :] + bias[c] ) * gate[b, c],
 *     b = r / rows_per_batch  (gate NULL: x[r, c] + bf16(...)),
 * the product and the sum rounded once each in float32.  Replaces the
 * reference's output projections with their residual updates: the
 * self-attention's `x + self.o(y) * e[2]` (model.py:175-176, :258-259), the
 * cross-attention's `x + cross_attn(...)` (:262 with the o-projection :188)
 * and the FFN's `x + ffn(...) * e[5]` (:263-265); the nn.Linear runs in
 * bf16 under autocast (float32 accumulation and bias, one rounding to bf16).
 * The bf16 layer output never reaches memory.  tcgen05 GEMM on SM pairs
 * (256 x 256 output tiles, persistent), float32 accumulation in TMEM.
 *   a:    bf16 [M, lda] (K columns used);  w: bf16 [N, ldw] (nn.Linear weight)
 *   bias: bf16 [N] or NULL;  x: float32 [M, ldx], updated in place
 *   gate: float32, row b at b * gate_batch_stride, or NULL
 * N must be a multiple of 32, K and lda / ldw multiples of 8, ldx and
 * gate_batch_stride multiples of 4; buffers 16-byte aligned.
 */
ICSA_API int icsa_dit_linear_residual(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                                      float* x, int64_t ldx, int M, int N, int K, int rows_per_batch,
                                      const float* gate, int64_t gate_batch_stride, cudaStream_t stream);

/*
 * Softmax attention of q over k, v with the default 1/sqrt(D) scale and no
 * mask: the DiT's cross-attention over the text tokens.  Replaces the
 * reference's flash_attention call (wanx/attention.py:18-85) made by
 * WanT2VCrossAttention (model.py:180-188; flash-attn's kernel in the
 * reference).  It runs the same tcgen05 dense attention kernel as the flat
 * query blocks of icsa_forward (D = 128: SM pairs; D = 64: one SM per tile):
 * fp32 accumulation, P rounded to bf16 for P.V, output rounded once to bf16.
 *   q:   bf16 [B, Lq, H, D], consecutive tokens q_row_stride elements apart
 *        (batch stride Lq * q_row_stride)
 *   k,v: bf16 [B, Lk, H, D], row strides k_row_stride / v_row_stride (a k|v
 *        GEMM output [B*Lk, 2*H*D] gives v at base + H*D with stride 2*H*D)
 *   out: bf16 [B, Lq, H, D], contiguous
 * D must be 64 or 128; row strides multiples of 8 elements and >= H*D;
 * all buffers 16-byte aligned.  Allocates nothing.
 */
ICSA_API int icsa_dit_cross_attention(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride,
                                      const void* v, int64_t v_row_stride, void* out, int B, int Lq, int Lk, int H,
                                      int D, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ICSA_DIT_H_ */
