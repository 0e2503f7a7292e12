/*
 * icsa.h -- C ABI of the B200 (sm_100a) in-context sparse attention library
 * (libicsa.so).
 *
 * The library computes exactly what the reference's
 * `in_context_sparse_attention.editing_sparse_attention(q, k, v, t_seq_len,
 * s_seq_len, alpha_2, alpha_3, SPARSITY_RATIO, backend)` computes
 * (in_context_sparse_attention/editing_sparse_attention.py:67-232), with all
 * stages on the GPU.  The signatures take plain device pointers, sizes and a
 * cudaStream_t; no framework types cross this boundary.
 *
 * Conventions
 *   - q, k, v and the output are contiguous [B, S, H, D] device buffers.
 *   - Every call is asynchronous on `stream` and performs no host
 *     synchronisation; it can be captured into a CUDA graph.
 *   - icsa_select and icsa_attend (and so icsa_forward) run part of their
 *     kernels on a side stream of the library's own, forked from `stream`
 *     and joined back to it by events: work enqueued on `stream` after the
 *     call still runs after all of it.  Each device has a small pool of such
 *     side streams: calls on different caller streams use different ones,
 *     and a side stream that has joined a stream capture serves only calls
 *     of that capture until it ends, so eager calls on other streams (or
 *     other captures) may run while a capture is open.  The library creates
 *     the first side streams on the first such call on each device; make that
 *     first call before any stream capture.
 *   - Every function returns an icsa_status; on failure
 *     icsa_last_error() returns a message for the calling thread.
 *   - Scratch memory ("workspace") is provided by the caller; its size comes
 *     from icsa_workspace_size().  The caller owns inputs, output and
 *     workspace; the library allocates no device memory.
 */
#ifndef ICSA_H_
#define ICSA_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define ICSA_API __attribute__((visibility("default")))
#else
#define ICSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of the buffers crossing the boundary. */
enum icsa_dtype { ICSA_BF16 = 0, ICSA_F32 = 1 };

/* Status codes. */
enum icsa_status {
  ICSA_OK = 0,
  ICSA_ERR_INVALID = 1,      /* bad argument or shape (reference: assert / ValueError) */
  ICSA_ERR_UNSUPPORTED = 2,  /* valid, but outside this build's limits (e.g. D not 64/128) */
  ICSA_ERR_CUDA = 3,         /* CUDA runtime or driver error */
  ICSA_ERR_WORKSPACE = 4,    /* workspace smaller than icsa_workspace_size() */
  ICSA_ERR_DEVICE_TIMEOUT = 5 /* a device-side bounded wait gave up (reported by icsa_device_status) */
};

/* Alpha (the residual weight `alpha_2` of the reference) forms. */
enum icsa_alpha_mode { ICSA_ALPHA_SCALAR = 0, ICSA_ALPHA_TENSOR = 1 };

/*
 * Problem description.  Fill it with icsa_problem_init(), which derives the
 * block counts with the reference's formulas, then set the dtype / alpha
 * fields.
 */
typedef struct icsa_problem {
  /* shape */
  int B, S, H, D;
  int t_seq_len;            /* target-video tokens (reference t_seq_len)                 */
  /* derived counts (reference formulas, filled by icsa_problem_init) */
  int num_blocks;           /* NB = ceil(S / 64)                                :90      */
  int n_t;                  /* t_seq_len // 64                                  :126     */
  int n_s;                  /* NB - n_t                                         :127     */
  int topK;                 /* selected source blocks, n_s // 8 by default      :129     */
  int num_flat;             /* query blocks sent to dense attention, NB // 2    :170     */
  int k_sparsity;           /* max(1, int(n_t * SPARSITY_RATIO))                :164     */
  int tkv;                  /* t_seq_len + topK * 64                            :139     */
  int nkv;                  /* ceil(tkv / 64): blocks of the extended KV                  */
  int top_k;                /* max(1, int(SPARSITY_RATIO * nkv)) tilelang_host.py:171    */
  /* element types */
  int q_dtype, k_dtype, v_dtype, out_dtype;   /* enum icsa_dtype */
  int outc_bf16;            /* 1: compressed-attention output is rounded to bf16 (the
                               reference's out_compress dtype is bf16)                   */
  /* alpha_2 */
  int alpha_mode;           /* enum icsa_alpha_mode                                       */
  int alpha_dtype;          /* enum icsa_dtype, tensor mode only                          */
  float alpha_scalar;       /* scalar mode                                                */
  int64_t alpha_strides[4]; /* tensor mode: element strides over [B,S,H,D], 0 = broadcast */
  int ca_bf16;              /* 1: out_compress*alpha is computed in bf16                  */
  /* options */
  int debug_keys;           /* no effect on the layout: the per-block selection scores
                               are always in the workspace (blockscore); kept so that
                               callers that set it keep working                         */
} icsa_problem;

/* Byte offsets of the named regions inside the workspace (for tests and
 * stage-by-stage callers). */
typedef struct icsa_workspace_layout {
  size_t total;
  size_t err;        /* int32 device status word                                   */
  size_t qsum, ksum, vsum;       /* bf16 [B*H, NB, D] block sums of bf16 values      */
  size_t qmean, kmean, vmean;    /* f32  [B*H, NB, D] block means                    */
  size_t scores;     /* f32 [B*H, NB, NB] compressed scores (q.k / sqrt(D))         */
  size_t rowmax, rowsum;         /* f32 [B*H, NB] softmax statistics               */
  size_t sharp;      /* f32 [B*H, NB] sharpness keys                                 */
  size_t colsum;     /* f32 [B*H, n_s] in-context relevance keys                     */
  size_t outc;       /* f32 [B*H, NB, D] compressed attention output                 */
  size_t sel;        /* i32 [B*H, topK] selected source blocks, by descending key    */
  size_t order;      /* i32 [B*H, NB] query blocks by descending sharpness           */
  size_t kv_rows;    /* i32 [B*H, nkv] first row of each extended-KV block           */
  size_t kc, vc;     /* bf16 [B*H, nkv_pad, D] extended-KV block sums                */
  size_t sparse_idx; /* i32 [B*H, n_sparse, top_k] exact blocks per sparse q block  */
  size_t sel_mask;   /* u32 [B*H, n_sparse, nkv_pad/32] same, as a bit set           */
  size_t blockscore; /* f32 [B*H, n_sparse, nkv] per-sparse-block scores QC . KC^T   */
  size_t qbf, kbf, vbf;          /* bf16 [B,S,H,D] copies of f32 inputs (else 0)    */
  size_t newk, newv; /* bf16 [B, nkv*64, H, D] extended KV when t_seq_len % 64 != 0 */
  int nkv_pad;       /* nkv rounded up to a multiple of 128                          */
  int n_sparse;      /* NB - num_flat                                               */
} icsa_workspace_layout;

/* Message describing the last failure on the calling thread. */
ICSA_API const char* icsa_last_error(void);

/* Library build string (architecture, version). */
ICSA_API const char* icsa_version(void);

/*
 * Fill `p` for q/k/v of shape [B,S,H,D].  Derived counts follow the
 * reference: editing_sparse_attention.py:90,126-129,139,164,170 and
 * tilelang_host.py:151-171.  select_ratio = 0.125 and flat_ratio = 0.5 give
 * the reference's hard-coded n_s // 8 and NB // 2.  Defaults: bf16 in/out,
 * scalar alpha 1.0, out_compress in bf16.
 */
ICSA_API int icsa_problem_init(icsa_problem* p, int B, int S, int H, int D, int t_seq_len, double sparsity_ratio,
                      double select_ratio, double flat_ratio);

/* Workspace bytes needed by icsa_forward for `p` (0 on invalid input). */
ICSA_API size_t icsa_workspace_size(const icsa_problem* p);

/* Region offsets of the workspace for `p`. */
ICSA_API int icsa_get_workspace_layout(const icsa_problem* p, icsa_workspace_layout* out);

/*
 * Whole call.  Replaces editing_sparse_attention()
 * (in_context_sparse_attention/editing_sparse_attention.py:67-232) with the
 * tilelang backend (tilelang_host.py:229-274 -> tilelang_kernels.py:681-997)
 * and the flash-attn dense part (:211-215).
 *   alpha: device pointer for ICSA_ALPHA_TENSOR, ignored for scalar mode.
 *   out:   [B,S,H,D] of p->out_dtype.
 */
ICSA_API int icsa_forward(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha, void* out,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Stage 1: block pooling.  Replaces compress_seq / the q_compress expression
 * (editing_sparse_attention.py:37-55,107-111) and the reduce kernels
 * reduce_q_kernel / reduce_kv_kernel (tilelang_kernels.py:33-120).
 */
ICSA_API int icsa_pool(const icsa_problem* p, const void* q, const void* k, const void* v, void* workspace,
              size_t workspace_bytes, cudaStream_t stream);

/*
 * Stage 2: compressed attention, in-context source-block retrieval,
 * sharpness split and per-block top-k.  Replaces torch_attention and the
 * selection code (editing_sparse_attention.py:58-64,113-172) and the host
 * top-k of the sparse backend (tilelang_host.py:170-173).  Needs stage 1.
 */
ICSA_API int icsa_select(const icsa_problem* p, const void* k, const void* v, void* workspace, size_t workspace_bytes,
                cudaStream_t stream);

/*
 * Stage 3: dense attention for the flat query blocks, block-sparse attention
 * with the interval term for the others, scatter and residual.  Replaces the
 * sparse kernel (tilelang_kernels.py:681-997), flash_attn_func
 * (editing_sparse_attention.py:211-215) and :217-232.  Needs stage 2.
 */
ICSA_API int icsa_attend(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha, void* out,
                void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * The two halves of stage 3, for per-kernel timing: icsa_attend_dense runs
 * the dense attention of the flat query blocks (the flash_attn_func call,
 * editing_sparse_attention.py:211-215, with its scatter and residual,
 * :217-232); icsa_attend_sparse the block-sparse attention of the remaining
 * blocks (tilelang_kernels.py:681-997 with the same epilogue).  Each writes
 * only its own query blocks of `out`; together they equal icsa_attend.
 */
ICSA_API int icsa_attend_dense(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha,
                               void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);
ICSA_API int icsa_attend_sparse(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha,
                                void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * The whole call with q, k, v and the output in HOST memory (pinned for
 * asynchronous copies), streamed through the current device by groups of
 * `group_heads` heads (a divisor of H): the copy of one group to the device,
 * the computation of another and the copy back of a third overlap on three
 * streams.  Every stage of the reference is independent per (batch, head)
 * (editing_sparse_attention.py:133-135,165-172; tilelang_kernels.py:802), so
 * the result equals icsa_forward on device copies of the same inputs.  No
 * counterpart in the reference, whose call takes device tensors.
 *   alpha:     device pointer for ICSA_ALPHA_TENSOR (strides over [B,S,H,D]).
 *   workspace: device memory of icsa_host_workspace_size() bytes, 256-byte
 *              aligned; icsa_device_status(workspace, ...) reports device
 *              timeouts of any group.
 * Returns after enqueueing; `stream` completes when the whole output is in
 * host memory.  Calls on one device are serialised by the library.
 */
ICSA_API size_t icsa_host_workspace_size(const icsa_problem* p, int group_heads);
ICSA_API int icsa_forward_host(const icsa_problem* p, int group_heads, const void* q, const void* k, const void* v,
                               const void* alpha, void* out, void* workspace, size_t workspace_bytes,
                               cudaStream_t stream);

/*
 * Synchronises `stream` and returns ICSA_OK or the status a device-side
 * bounded wait recorded in the workspace during the preceding calls.
 */
ICSA_API int icsa_device_status(void* workspace, cudaStream_t stream);

/*
 * Per-device record of device-side timeouts, for callers that no longer hold
 * the workspace of the calls they made (no counterpart in the reference,
 * whose host asserts and raises: tilelang_host.py:251-260,
 * editing_sparse_attention.py:31-34).  Every bounded wait that gives up also
 * writes its code into a status word of the current device that outlives the
 * call.  This function synchronises `stream`, then returns ICSA_OK if no wait
 * on the current device gave up since the record was last cleared, else
 * ICSA_ERR_DEVICE_TIMEOUT (with the code in icsa_last_error()).  With
 * `clear` != 0 it clears the record.  It synchronises, so it cannot be
 * captured in a CUDA graph; call it after a graph replay instead.
 */
ICSA_API int icsa_last_status(cudaStream_t stream, int clear);

/*
 * Self-test of the device-side bounded waits (no counterpart in the
 * reference): launches a kernel whose mbarrier wait can never complete; the
 * wait gives up after about one second, records a status code in the first
 * word of `workspace` and returns, after which icsa_device_status(workspace)
 * reports ICSA_ERR_DEVICE_TIMEOUT and the context stays usable.  Needs at
 * least 256 bytes of device workspace.
 */
ICSA_API int icsa_wait_selftest(void* workspace, cudaStream_t stream);

/*
 * Allocation-free variant of icsa_forward.  This entry point has no
 * counterpart in the reference; it exists for callers that cannot allocate
 * device memory where they make the call (a plugin host that owns all
 * allocations, a runtime with a fixed memory budget, an FFI caller without a
 * CUDA allocator).  They pass inputs and output only; the scratch is a
 * 64 MiB array inside the library's device code, which each GPU that loads it
 * keeps until the process exits (loaded at the first call on that GPU under
 * the default lazy module loading).  Problems whose icsa_workspace_size()
 * exceeds icsa_static_scratch_bytes() are rejected with ICSA_ERR_WORKSPACE.
 * All calls share that one array: calls that overlap on the GPU race, so
 * order them on one stream.  The first call on each device looks the array's
 * address up (and may load the module); make it before any stream capture.
 * The address is kept per CUDA context: after a cudaDeviceReset() the next
 * call looks it up again in the new context.
 * No cudaMalloc/cudaFree or other allocating routine is called.
 */
ICSA_API int icsa_forward_static(const icsa_problem* p, const void* q, const void* k, const void* v,
                                 const void* alpha, void* out, cudaStream_t stream);

/* Size in bytes of the static scratch used by icsa_forward_static. */
ICSA_API size_t icsa_static_scratch_bytes(void);

/*
 * icsa_device_status for the static scratch of icsa_forward_static: waits
 * for `stream` and returns ICSA_OK, or ICSA_ERR_DEVICE_TIMEOUT if a
 * device-side bounded wait of the preceding icsa_forward_static calls on the
 * current device gave up.  Like icsa_forward_static it allocates nothing.
 */
ICSA_API int icsa_static_device_status(cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ICSA_H_ */
