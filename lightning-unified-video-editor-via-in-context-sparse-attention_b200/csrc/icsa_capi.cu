// C ABI of libicsa.so: argument checking, workspace layout, TMA descriptor
// construction and the stage sequence of one call.  Declarations and the
// reference interfaces each entry point replaces are in include/icsa.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cmath>
#include <string>
#include <algorithm>
#include <mutex>

#include "icsa_kernels.cuh"
#include "icsa_dit.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(ICSA_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// ---------------------------------------------------------------------------
// Validation of a problem description.
// ---------------------------------------------------------------------------
int check_problem(const icsa_problem* p) {
  if (p == nullptr) return fail(ICSA_ERR_INVALID, "problem is NULL");
  if (p->B < 1 || p->S < 1 || p->H < 1) return fail(ICSA_ERR_INVALID, "B, S, H must be positive (got %d, %d, %d)", p->B, p->S, p->H);
  if (p->D != 64 && p->D != 128) return fail(ICSA_ERR_UNSUPPORTED, "head dim D=%d: this build supports D in {64, 128}", p->D);
  if (p->t_seq_len < 0 || p->t_seq_len > p->S)
    return fail(ICSA_ERR_INVALID, "t_seq_len=%d must lie in [0, S=%d]", p->t_seq_len, p->S);
  const int NB = (p->S + icsa::kBlock - 1) / icsa::kBlock;
  if (p->num_blocks != NB || p->n_t != p->t_seq_len / icsa::kBlock || p->n_s != NB - p->n_t)
    return fail(ICSA_ERR_INVALID, "derived block counts are inconsistent; fill the problem with icsa_problem_init");
  if (p->topK < 0 || p->topK > p->n_s) return fail(ICSA_ERR_INVALID, "topK=%d exceeds the %d source blocks", p->topK, p->n_s);
  if (p->num_flat < 0 || p->num_flat > NB) return fail(ICSA_ERR_INVALID, "num_flat=%d must lie in [0, %d]", p->num_flat, NB);
  if (p->tkv != p->t_seq_len + p->topK * icsa::kBlock || p->nkv != (p->tkv + icsa::kBlock - 1) / icsa::kBlock)
    return fail(ICSA_ERR_INVALID, "tkv / nkv inconsistent with t_seq_len and topK");
  if (p->nkv < 1) return fail(ICSA_ERR_INVALID, "the extended KV is empty (t_seq_len // 64 == 0 and no source block selected)");
  if (p->top_k < 1 || p->top_k > p->nkv)
    return fail(ICSA_ERR_INVALID, "top_k=%d must lie in [1, nkv=%d] (torch.topk would fail)", p->top_k, p->nkv);
  if (p->k_sparsity < 1) return fail(ICSA_ERR_INVALID, "k_sparsity must be >= 1");
  auto dt_ok = [](int d) { return d == ICSA_BF16 || d == ICSA_F32; };
  if (!dt_ok(p->q_dtype) || !dt_ok(p->k_dtype) || !dt_ok(p->v_dtype) || !dt_ok(p->out_dtype))
    return fail(ICSA_ERR_INVALID, "dtype codes must be ICSA_BF16 or ICSA_F32");
  if (p->alpha_mode != ICSA_ALPHA_SCALAR && p->alpha_mode != ICSA_ALPHA_TENSOR)
    return fail(ICSA_ERR_INVALID, "alpha_mode must be ICSA_ALPHA_SCALAR or ICSA_ALPHA_TENSOR");
  if (p->alpha_mode == ICSA_ALPHA_TENSOR && !dt_ok(p->alpha_dtype))
    return fail(ICSA_ERR_INVALID, "alpha_dtype must be ICSA_BF16 or ICSA_F32");
  if (NB > 16384 || p->nkv > 16384)
    return fail(ICSA_ERR_UNSUPPORTED, "NB=%d / nkv=%d exceed this build's limit of 16384 blocks", NB, p->nkv);
  return ICSA_OK;
}

void compute_layout(const icsa_problem* p, icsa_workspace_layout* w) {
  std::memset(w, 0, sizeof(*w));
  const size_t BH = size_t(p->B) * p->H, NB = p->num_blocks, D = p->D;
  const int nkv_pad = round_up(p->nkv, 128);
  const int n_sparse = p->num_blocks - p->num_flat;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + (bytes == 0 ? 1 : bytes));
    return o;
  };
  w->err = take(256);
  w->qsum = take(BH * NB * D * 2);
  w->ksum = take(BH * NB * D * 2);
  w->vsum = take(BH * NB * D * 2);
  w->qmean = take(BH * NB * D * 4);
  w->kmean = take(BH * NB * D * 4);
  w->vmean = take(BH * NB * D * 4);
  w->scores = take(BH * NB * NB * 4);
  w->rowmax = take(BH * NB * 4);
  w->rowsum = take(BH * NB * 4);
  w->sharp = take(BH * NB * 4);
  w->colsum = take(BH * size_t(p->n_s) * 4);
  w->outc = take(BH * NB * D * 4);
  w->sel = take(BH * size_t(p->topK) * 4);
  w->order = take(BH * NB * 4);
  w->kv_rows = take(BH * size_t(p->nkv) * 4);
  w->kc = take(BH * size_t(nkv_pad) * D * 2);
  w->vc = take(BH * size_t(nkv_pad) * D * 2);
  w->sparse_idx = take(BH * size_t(n_sparse) * p->top_k * 4);
  w->sel_mask = take(BH * size_t(n_sparse) * (nkv_pad / 32) * 4);
  w->blockscore = take(BH * size_t(n_sparse) * p->nkv * 4);
  const size_t act = size_t(p->B) * p->S * p->H * D * 2;
  w->qbf = p->q_dtype == ICSA_F32 ? take(act) : 0;
  w->kbf = p->k_dtype == ICSA_F32 ? take(act) : 0;
  w->vbf = p->v_dtype == ICSA_F32 ? take(act) : 0;
  const bool aligned = (p->t_seq_len % icsa::kBlock) == 0;
  const size_t ext = size_t(p->B) * p->nkv * icsa::kBlock * p->H * D * 2;
  w->newk = aligned ? 0 : take(ext);
  w->newv = aligned ? 0 : take(ext);
  w->total = off;
  w->nkv_pad = nkv_pad;
  w->n_sparse = n_sparse;
}

// ---------------------------------------------------------------------------
// TMA descriptors.  cuTensorMapEncodeTiled is fetched from the driver through
// the runtime, so the library does not link against libcuda directly.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// bf16 [B, rows, H, D] with a {64, 1, 64, 1} box (64 features x 64 rows);
// consecutive rows `row_stride` elements apart (H * D when contiguous).
int encode_rows_map(CUtensorMap* m, const void* base, int B, int rows, int H, int D, int64_t row_stride = 0) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t rs = row_stride > 0 ? cuuint64_t(row_stride) : cuuint64_t(H) * D;
  const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(rows), cuuint64_t(B)};
  const cuuint64_t strides[3] = {cuuint64_t(D) * 2, rs * 2, cuuint64_t(rows) * rs * 2};
  const cuuint32_t box[4] = {64, 1, 64, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled (rows map) failed with %d", int(r));
  return ICSA_OK;
}

// bf16 [rows, cols] row-major with leading dimension ld (elements), box
// {64, 128}: 128 rows x 64 columns (one 128-byte swizzled row each).
int encode_matrix_map(CUtensorMap* m, const void* base, int rows, int cols, int64_t ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled (matrix map) failed with %d", int(r));
  return ICSA_OK;
}

// bf16 [BH, n, D] with a {64, 128, 1} box (64 features x 128 pooled rows).
int encode_pooled_map(CUtensorMap* m, const void* base, int BH, int n, int D) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(n), cuuint64_t(BH)};
  const cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(n) * D * 2};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ICSA_ERR_CUDA, "cuTensorMapEncodeTiled (pooled map) failed with %d", int(r));
  return ICSA_OK;
}

}  // namespace

// ===========================================================================
// Stage drivers
// ===========================================================================
namespace {

template <typename T>
T* at(void* ws, size_t off) {
  return off == 0 ? nullptr : reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off);
}

int check_call(const icsa_problem* p, void* ws, size_t ws_bytes, icsa_workspace_layout* L) {
  int rc = check_problem(p);
  if (rc != ICSA_OK) return rc;
  compute_layout(p, L);
  if (ws == nullptr) return fail(ICSA_ERR_INVALID, "workspace is NULL");
  if (ws_bytes < L->total)
    return fail(ICSA_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu bytes required", ws_bytes, L->total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return fail(ICSA_ERR_INVALID, "workspace must be 256-byte aligned");
  return ICSA_OK;
}

// ---------------------------------------------------------------------------
// Side streams for the parts of one call that may run side by side:
// out_compress beside the selection chain, and the block-sparse attention
// beside the dense attention (its CTAs take the SMs that the dense kernel's
// last wave leaves idle).  Side work is ordered by events: the side stream
// waits for an event recorded on the caller's stream, and the caller's stream
// waits for an event recorded after the side work, so the caller sees one
// ordered call and a captured caller stream captures the side work too.
//
// Each device has a small pool of side streams (each with its own two
// events).  A call takes the side stream that last served its caller stream
// when that one is free for it, else the least recently used free one:
// * a side stream that has joined a stream capture stays inside it until the
//   capture ends, so while a capture is open it serves only calls of that
//   same capture; eager calls, and other captures, take another one;
// * eager calls on different caller streams get different side streams (up
//   to kMaxSides per device), so they are not serialised behind each other.
// kPrecreated side streams are created by the first call on a device; more
// are created on demand, which a call inside a capture cannot always do
// (stream creation is refused in some capture modes), hence the first call
// on a device belongs outside any capture.  The mutex keeps host threads from
// interleaving their use of one side stream's events.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
constexpr int kPrecreated = 2, kMaxSides = 8;

struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  cudaStream_t owner = nullptr;  // caller stream it served last
  uint64_t last_use = 0;
};
struct DeviceSides {
  SideStream pool[kMaxSides];
  int count = 0;
  uint64_t tick = 0;
};
std::mutex g_side_mutex;
DeviceSides g_side[kMaxDevices];

int create_side(SideStream* s) {
  cudaError_t e;
  if ((e = cudaEventCreateWithFlags(&s->fork, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&s->join, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e, "side stream / event creation (make the first call on a device outside stream capture)");
  return ICSA_OK;
}

// Capture state of a stream: 0 idle, 1 inside capture `*id`, -1 inside an
// invalidated capture (busy until that capture ends).
int capture_state(cudaStream_t s, unsigned long long* id) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  *id = 0;
  if (cudaStreamGetCaptureInfo(s, &st, id) != cudaSuccess) return -1;
  return st == cudaStreamCaptureStatusNone ? 0 : st == cudaStreamCaptureStatusActive ? 1 : -1;
}

// Called with g_side_mutex held: a side stream for work forked from `caller`.
int side_stream(cudaStream_t caller, SideStream** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(ICSA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  DeviceSides& d = g_side[dev];
  while (d.count < kPrecreated) {
    const int rc = create_side(&d.pool[d.count]);
    if (rc != ICSA_OK) return rc;
    ++d.count;
  }
  unsigned long long cid = 0;
  const int cstate = capture_state(caller, &cid);
  if (cstate < 0) return fail(ICSA_ERR_CUDA, "the caller's stream is inside an invalidated stream capture");
  // usable: idle, or already inside the caller's own capture
  auto usable = [&](SideStream& s) {
    unsigned long long sid = 0;
    const int st = capture_state(s.stream, &sid);
    return st == 0 || (st == 1 && cstate == 1 && sid == cid);
  };
  SideStream* pick = nullptr;
  for (int i = 0; i < d.count && pick == nullptr; ++i)
    if (d.pool[i].owner == caller && usable(d.pool[i])) pick = &d.pool[i];
  if (pick == nullptr) {
    // a side stream no other caller has claimed yet, else the least recently used usable one
    for (int i = 0; i < d.count && pick == nullptr; ++i)
      if (d.pool[i].owner == nullptr && usable(d.pool[i])) pick = &d.pool[i];
    if (pick == nullptr && d.count < kMaxSides) {
      const int rc = create_side(&d.pool[d.count]);
      if (rc != ICSA_OK) return rc;
      pick = &d.pool[d.count++];
    }
    if (pick == nullptr)
      for (int i = 0; i < d.count; ++i)
        if (usable(d.pool[i]) && (pick == nullptr || d.pool[i].last_use < pick->last_use)) pick = &d.pool[i];
  }
  if (pick == nullptr)
    return fail(ICSA_ERR_UNSUPPORTED, "all %d side streams of device %d are inside other stream captures", d.count, dev);
  pick->owner = caller;
  pick->last_use = ++d.tick;
  *out = pick;
  return ICSA_OK;
}

// side waits for the work enqueued on `stream` so far
int fork_to(const SideStream* s, cudaStream_t stream) {
  cudaError_t e = cudaEventRecord(s->fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s->stream, s->fork, 0);
  return e == cudaSuccess ? ICSA_OK : cuda_fail(e, "fork to the side stream");
}

// `stream` waits for the work enqueued on the side stream so far
int join_from(const SideStream* s, cudaStream_t stream) {
  cudaError_t e = cudaEventRecord(s->join, s->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, s->join, 0);
  return e == cudaSuccess ? ICSA_OK : cuda_fail(e, "join from the side stream");
}

icsa::SelectParams make_select_params(const icsa_problem* p, const icsa_workspace_layout& L, void* ws, const void* k,
                                      const void* v) {
  icsa::SelectParams s;
  std::memset(&s, 0, sizeof(s));
  s.B = p->B; s.H = p->H; s.D = p->D; s.S = p->S;
  s.NB = p->num_blocks; s.n_t = p->n_t; s.n_s = p->n_s; s.topK = p->topK; s.num_flat = p->num_flat;
  s.n_sparse = L.n_sparse; s.k_sparsity = p->k_sparsity; s.top_k = p->top_k;
  s.nkv = p->nkv; s.nkv_pad = L.nkv_pad; s.tkv = p->tkv; s.t_seq_len = p->t_seq_len;
  s.inv_sqrt_d_div = float(std::sqrt(double(p->D)));
  s.qmean = at<float>(ws, L.qmean); s.kmean = at<float>(ws, L.kmean); s.vmean = at<float>(ws, L.vmean);
  s.qsum = at<__nv_bfloat16>(ws, L.qsum); s.ksum = at<__nv_bfloat16>(ws, L.ksum); s.vsum = at<__nv_bfloat16>(ws, L.vsum);
  s.scores = at<float>(ws, L.scores); s.rowmax = at<float>(ws, L.rowmax); s.rowsum = at<float>(ws, L.rowsum);
  s.sharp = at<float>(ws, L.sharp); s.colsum = at<float>(ws, L.colsum); s.outc = at<float>(ws, L.outc);
  s.sel = at<int>(ws, L.sel); s.order = at<int>(ws, L.order); s.kv_rows = at<int>(ws, L.kv_rows);
  s.kc = at<__nv_bfloat16>(ws, L.kc); s.vc = at<__nv_bfloat16>(ws, L.vc);
  s.sparse_idx = at<int>(ws, L.sparse_idx); s.sel_mask = at<uint32_t>(ws, L.sel_mask);
  s.blockscore = at<float>(ws, L.blockscore);
  s.k_src = p->k_dtype == ICSA_F32 ? at<__nv_bfloat16>(ws, L.kbf) : static_cast<const __nv_bfloat16*>(k);
  s.v_src = p->v_dtype == ICSA_F32 ? at<__nv_bfloat16>(ws, L.vbf) : static_cast<const __nv_bfloat16*>(v);
  s.newk = at<__nv_bfloat16>(ws, L.newk); s.newv = at<__nv_bfloat16>(ws, L.newv);
  // the pool stage rounds the means to bf16 for bf16 inputs and for f32
  // inputs whose compressed attention runs in bf16
  s.means_bf16 = (p->q_dtype == ICSA_BF16 || p->outc_bf16) && (p->k_dtype == ICSA_BF16 || p->outc_bf16);
  s.vmean_bf16 = p->v_dtype == ICSA_BF16 || p->outc_bf16;
  s.err = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + L.err);
  return s;
}

int run_pool(const icsa_problem* p, const icsa_workspace_layout& L, void* ws, const void* q, const void* k,
             const void* v, cudaStream_t stream) {
  icsa::PoolParams pp;
  std::memset(&pp, 0, sizeof(pp));
  pp.B = p->B; pp.S = p->S; pp.H = p->H; pp.D = p->D;
  pp.num_blocks = p->num_blocks; pp.block_stride = p->num_blocks;
  const void* xs[3] = {q, k, v};
  const int dts[3] = {p->q_dtype, p->k_dtype, p->v_dtype};
  const size_t sums[3] = {L.qsum, L.ksum, L.vsum}, means[3] = {L.qmean, L.kmean, L.vmean}, cps[3] = {L.qbf, L.kbf, L.vbf};
  for (int i = 0; i < 3; ++i) {
    pp.t[i].x = xs[i];
    pp.t[i].dtype = dts[i];
    pp.t[i].sum_bf16 = at<__nv_bfloat16>(ws, sums[i]);
    pp.t[i].mean_f32 = at<float>(ws, means[i]);
    pp.t[i].copy_bf16 = at<__nv_bfloat16>(ws, cps[i]);
    pp.t[i].round_mean_bf16 = p->outc_bf16;
  }
  cudaError_t e = icsa::launch_pool(pp, stream);
  return e == cudaSuccess ? ICSA_OK : cuda_fail(e, "pool");
}

// The selection chain after the row statistics (column sums, the two sorts,
// the extended KV and the per-block top-k), on `stream`.
int run_selection_chain(const icsa_problem* p, const icsa_workspace_layout& L, const icsa::SelectParams& s,
                        cudaStream_t stream) {
  cudaError_t e = icsa::launch_colsum(s, stream);
  if (e != cudaSuccess) return cuda_fail(e, "column sums");
  e = icsa::launch_selection(s, stream);
  if (e != cudaSuccess) return cuda_fail(e, "block selection");
  e = icsa::launch_extended_kv(s, stream);
  if (e != cudaSuccess) return cuda_fail(e, "extended KV");
  if (p->t_seq_len % icsa::kBlock != 0) {
    // pool the materialised extended K/V into the sparse-level block sums
    icsa::PoolParams pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.B = p->B; pp.S = p->nkv * icsa::kBlock; pp.H = p->H; pp.D = p->D;
    pp.num_blocks = p->nkv; pp.block_stride = L.nkv_pad;
    pp.t[1].x = s.newk; pp.t[1].dtype = ICSA_BF16; pp.t[1].sum_bf16 = s.kc;
    pp.t[2].x = s.newv; pp.t[2].dtype = ICSA_BF16; pp.t[2].sum_bf16 = s.vc;
    e = icsa::launch_pool(pp, stream);
    if (e != cudaSuccess) return cuda_fail(e, "extended KV pooling");
  }
  e = icsa::launch_sparse_topk(s, stream);
  if (e != cudaSuccess) return cuda_fail(e, "sparse top-k");
  return ICSA_OK;
}

int run_select(const icsa_problem* p, const icsa_workspace_layout& L, void* ws, const void* k, const void* v,
               cudaStream_t stream) {
  icsa::SelectParams s = make_select_params(p, L, ws, k, v);
  cudaError_t e = icsa::launch_compressed_scores(s, stream);
  if (e != cudaSuccess) return cuda_fail(e, "compressed scores");
  // out_compress is read only by the attention epilogue: it runs on the side
  // stream beside the selection chain
  std::lock_guard<std::mutex> lock(g_side_mutex);
  SideStream* side = nullptr;
  int rc = side_stream(stream, &side);
  if (rc == ICSA_OK) rc = fork_to(side, stream);
  if (rc != ICSA_OK) return rc;
  e = icsa::launch_outc(s, side->stream);
  rc = e == cudaSuccess ? run_selection_chain(p, L, s, stream) : cuda_fail(e, "out_compress");
  const int jrc = join_from(side, stream);
  return rc != ICSA_OK ? rc : jrc;
}

constexpr int kAttendDense = 1, kAttendSparse = 2;

int run_attend(const icsa_problem* p, const icsa_workspace_layout& L, void* ws, const void* q, const void* k,
               const void* v, const void* alpha, void* out, cudaStream_t stream,
               int parts = kAttendDense | kAttendSparse) {
  if (out == nullptr) return fail(ICSA_ERR_INVALID, "output pointer is NULL");
  if (p->alpha_mode == ICSA_ALPHA_TENSOR && alpha == nullptr) return fail(ICSA_ERR_INVALID, "alpha tensor is NULL");
  const bool aligned = (p->t_seq_len % icsa::kBlock) == 0;
  const void* qb = p->q_dtype == ICSA_F32 ? at<void>(ws, L.qbf) : q;
  const void* kb = aligned ? (p->k_dtype == ICSA_F32 ? at<void>(ws, L.kbf) : k) : at<void>(ws, L.newk);
  const void* vb = aligned ? (p->v_dtype == ICSA_F32 ? at<void>(ws, L.vbf) : v) : at<void>(ws, L.newv);
  const int kv_rows = aligned ? p->S : p->nkv * icsa::kBlock;
  icsa::AttnMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  const int BH = p->B * p->H;
  int rc;
  if ((rc = encode_rows_map(&maps.q, qb, p->B, p->S, p->H, p->D)) != ICSA_OK) return rc;
  if ((rc = encode_rows_map(&maps.k, kb, p->B, kv_rows, p->H, p->D)) != ICSA_OK) return rc;
  if ((rc = encode_rows_map(&maps.v, vb, p->B, kv_rows, p->H, p->D)) != ICSA_OK) return rc;
  if ((rc = encode_pooled_map(&maps.kc, at<void>(ws, L.kc), BH, L.nkv_pad, p->D)) != ICSA_OK) return rc;
  if ((rc = encode_pooled_map(&maps.vc, at<void>(ws, L.vc), BH, L.nkv_pad, p->D)) != ICSA_OK) return rc;

  icsa::AttnParams a;
  std::memset(&a, 0, sizeof(a));
  a.B = p->B; a.S = p->S; a.H = p->H; a.NB = p->num_blocks;
  a.num_flat = p->num_flat; a.n_sparse = L.n_sparse;
  a.flat_tiles = (p->num_flat + 1) / 2; a.sparse_tiles = (L.n_sparse + 1) / 2;
  a.nkv = p->nkv; a.nkv_pad = L.nkv_pad; a.tkv = p->tkv; a.top_k = p->top_k;
  a.scale_log2 = float(std::sqrt(1.0 / p->D) * 1.44269504);
  a.order = at<int>(ws, L.order); a.kv_rows = at<int>(ws, L.kv_rows);
  a.sparse_idx = at<int>(ws, L.sparse_idx); a.sel_mask = at<uint32_t>(ws, L.sel_mask);
  a.outc = at<float>(ws, L.outc); a.outc_bf16 = p->outc_bf16;
  a.alpha_mode = p->alpha_mode; a.alpha_dtype = p->alpha_dtype; a.ca_bf16 = p->ca_bf16;
  a.alpha_scalar = p->alpha_scalar; a.alpha = alpha;
  for (int i = 0; i < 4; ++i) a.alpha_strides[i] = p->alpha_strides[i];
  a.out = out; a.out_dtype = p->out_dtype;
  // bf16 output from a 16-byte aligned pointer: written by TMA stores
  if (p->out_dtype == ICSA_BF16 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    if ((rc = encode_rows_map(&maps.o, out, p->B, p->S, p->H, p->D)) != ICSA_OK) return rc;
    a.out_tma = 1;
  }
  a.err = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + L.err);
  if (parts == (kAttendDense | kAttendSparse) && p->num_flat > 0 && L.n_sparse > 0) {
    // both halves: the dense attention is launched first on the caller's
    // stream and the block-sparse attention on the side stream, so the
    // sparse CTAs fill the SMs that the dense kernel's last wave leaves idle
    std::lock_guard<std::mutex> lock(g_side_mutex);
    SideStream* side = nullptr;
    if ((rc = side_stream(stream, &side)) != ICSA_OK || (rc = fork_to(side, stream)) != ICSA_OK) return rc;
    cudaError_t e = icsa::launch_flat_attention(a, maps, p->D, stream);
    rc = e == cudaSuccess ? ICSA_OK : cuda_fail(e, "dense attention");
    if (rc == ICSA_OK) {
      e = icsa::launch_sparse_attention(a, maps, p->D, side->stream);
      if (e != cudaSuccess) rc = cuda_fail(e, "sparse attention");
    }
    const int jrc = join_from(side, stream);
    return rc != ICSA_OK ? rc : jrc;
  }
  if (parts & kAttendDense) {
    cudaError_t e = icsa::launch_flat_attention(a, maps, p->D, stream);
    if (e != cudaSuccess) return cuda_fail(e, "dense attention");
  }
  if (parts & kAttendSparse) {
    cudaError_t e = icsa::launch_sparse_attention(a, maps, p->D, stream);
    if (e != cudaSuccess) return cuda_fail(e, "sparse attention");
  }
  return ICSA_OK;
}

}  // namespace

// ===========================================================================
// Exported C ABI
// ===========================================================================
extern "C" {

void icsa_set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

const char* icsa_last_error(void) { return g_last_error.c_str(); }

const char* icsa_version(void) { return "icsa-b200 0.1 (sm_100a, tcgen05)"; }

int icsa_problem_init(icsa_problem* p, int B, int S, int H, int D, int t_seq_len, double sparsity_ratio,
                      double select_ratio, double flat_ratio) {
  if (p == nullptr) return fail(ICSA_ERR_INVALID, "problem is NULL");
  std::memset(p, 0, sizeof(*p));
  if (B < 1 || S < 1 || H < 1) return fail(ICSA_ERR_INVALID, "B, S, H must be positive");
  if (t_seq_len < 0 || t_seq_len > S) return fail(ICSA_ERR_INVALID, "t_seq_len=%d must lie in [0, S=%d]", t_seq_len, S);
  if (!(sparsity_ratio >= 0.0) || !(select_ratio >= 0.0) || !(flat_ratio >= 0.0 && flat_ratio <= 1.0))
    return fail(ICSA_ERR_INVALID, "ratios must be non-negative and flat_ratio <= 1");
  p->B = B; p->S = S; p->H = H; p->D = D; p->t_seq_len = t_seq_len;
  p->num_blocks = (S + icsa::kBlock - 1) / icsa::kBlock;
  p->n_t = t_seq_len / icsa::kBlock;
  p->n_s = p->num_blocks - p->n_t;
  p->topK = int(double(p->n_s) * select_ratio);
  p->num_flat = int(double(p->num_blocks) * flat_ratio);
  p->k_sparsity = std::max(1, int(double(p->n_t) * sparsity_ratio));
  p->tkv = t_seq_len + p->topK * icsa::kBlock;
  p->nkv = (p->tkv + icsa::kBlock - 1) / icsa::kBlock;
  p->top_k = std::max(1, int(sparsity_ratio * double(p->nkv)));
  p->q_dtype = p->k_dtype = p->v_dtype = p->out_dtype = ICSA_BF16;
  p->outc_bf16 = 1;
  p->alpha_mode = ICSA_ALPHA_SCALAR;
  p->alpha_dtype = ICSA_F32;
  p->alpha_scalar = 1.0f;
  p->ca_bf16 = 1;
  return check_problem(p);
}

size_t icsa_workspace_size(const icsa_problem* p) {
  if (check_problem(p) != ICSA_OK) return 0;
  icsa_workspace_layout L;
  compute_layout(p, &L);
  return L.total;
}

int icsa_get_workspace_layout(const icsa_problem* p, icsa_workspace_layout* out) {
  int rc = check_problem(p);
  if (rc != ICSA_OK) return rc;
  if (out == nullptr) return fail(ICSA_ERR_INVALID, "layout output is NULL");
  compute_layout(p, out);
  return ICSA_OK;
}

int icsa_pool(const icsa_problem* p, const void* q, const void* k, const void* v, void* workspace,
              size_t workspace_bytes, cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "q, k and v must be non-NULL");
  cudaError_t e = cudaMemsetAsync(workspace, 0, 256, stream);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  return run_pool(p, L, workspace, q, k, v, stream);
}

int icsa_select(const icsa_problem* p, const void* k, const void* v, void* workspace, size_t workspace_bytes,
                cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "k and v must be non-NULL");
  return run_select(p, L, workspace, k, v, stream);
}

int icsa_attend(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha, void* out,
                void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "q, k and v must be non-NULL");
  return run_attend(p, L, workspace, q, k, v, alpha, out, stream);
}

int icsa_attend_dense(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha,
                      void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "q, k and v must be non-NULL");
  return run_attend(p, L, workspace, q, k, v, alpha, out, stream, kAttendDense);
}

int icsa_attend_sparse(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha,
                       void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "q, k and v must be non-NULL");
  return run_attend(p, L, workspace, q, k, v, alpha, out, stream, kAttendSparse);
}

int icsa_forward(const icsa_problem* p, const void* q, const void* k, const void* v, const void* alpha, void* out,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  icsa_workspace_layout L;
  int rc = check_call(p, workspace, workspace_bytes, &L);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr) return fail(ICSA_ERR_INVALID, "q, k and v must be non-NULL");
  cudaError_t e = cudaMemsetAsync(workspace, 0, 256, stream);
  if (e != cudaSuccess) return cuda_fail(e, "status reset");
  if ((rc = run_pool(p, L, workspace, q, k, v, stream)) != ICSA_OK) return rc;
  if ((rc = run_select(p, L, workspace, k, v, stream)) != ICSA_OK) return rc;
  return run_attend(p, L, workspace, q, k, v, alpha, out, stream);
}

int icsa_device_status(void* workspace, cudaStream_t stream) {
  if (workspace == nullptr) return fail(ICSA_ERR_INVALID, "workspace is NULL");
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  int code = 0;
  e = cudaMemcpy(&code, workspace, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (code != 0) return fail(ICSA_ERR_DEVICE_TIMEOUT, "a device-side wait gave up (code 0x%x)", code);
  return ICSA_OK;
}

int icsa_dit_cross_attention(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride,
                             const void* v, int64_t v_row_stride, void* out, int B, int Lq, int Lk, int H, int D,
                             cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(ICSA_ERR_INVALID, "cross attention: q, k, v and out must be non-NULL");
  if (B < 1 || Lq < 1 || Lk < 1 || H < 1)
    return fail(ICSA_ERR_INVALID, "cross attention: B, Lq, Lk, H must be positive (got %d, %d, %d, %d)", B, Lq, Lk, H);
  if (D != 64 && D != 128) return fail(ICSA_ERR_UNSUPPORTED, "cross attention: head dim D=%d (supported: 64, 128)", D);
  const int64_t hd = int64_t(H) * D;
  const int64_t strides[3] = {q_row_stride, k_row_stride, v_row_stride};
  for (int i = 0; i < 3; ++i)
    if (strides[i] < hd || strides[i] % 8 != 0)
      return fail(ICSA_ERR_INVALID, "cross attention: row strides must be multiples of 8 elements and >= H*D=%lld",
                  (long long)hd);
  const void* ptrs[4] = {q, k, v, out};
  for (int i = 0; i < 4; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0)
      return fail(ICSA_ERR_INVALID, "cross attention: buffers must be 16-byte aligned");
  const int nbq = (Lq + icsa::kBlock - 1) / icsa::kBlock, nbk = (Lk + icsa::kBlock - 1) / icsa::kBlock;
  if (nbq > (1 << 24) || nbk > 16384)
    return fail(ICSA_ERR_UNSUPPORTED, "cross attention: Lq=%d / Lk=%d exceed this build's limits", Lq, Lk);
  icsa::AttnMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  int rc;
  if ((rc = encode_rows_map(&maps.q, q, B, Lq, H, D, q_row_stride)) != ICSA_OK) return rc;
  if ((rc = encode_rows_map(&maps.k, k, B, Lk, H, D, k_row_stride)) != ICSA_OK) return rc;
  if ((rc = encode_rows_map(&maps.v, v, B, Lk, H, D, v_row_stride)) != ICSA_OK) return rc;
  if ((rc = encode_rows_map(&maps.o, out, B, Lq, H, D)) != ICSA_OK) return rc;
  // every query block is a "flat" block in its natural order, the keys are
  // the Lk rows of k / v (no order table, no block table), and there is no
  // residual term: the dense attention kernels compute softmax(q k^T / sqrt(D)) v
  icsa::AttnParams a;
  std::memset(&a, 0, sizeof(a));
  a.B = B; a.S = Lq; a.H = H; a.NB = nbq;
  a.num_flat = nbq; a.n_sparse = 0;
  a.flat_tiles = (nbq + 1) / 2; a.sparse_tiles = 0;
  a.nkv = nbk; a.nkv_pad = (nbk + 127) / 128 * 128; a.tkv = Lk; a.top_k = 0;
  a.scale_log2 = float(std::sqrt(1.0 / D) * 1.44269504);
  a.alpha_mode = ICSA_ALPHA_SCALAR; a.alpha_scalar = 0.f;
  a.out = out; a.out_dtype = ICSA_BF16; a.out_tma = 1;
  cudaError_t e = icsa::launch_flat_attention(a, maps, D, stream);
  return e == cudaSuccess ? ICSA_OK : cuda_fail(e, "cross attention");
}

int icsa_dit_linear_residual(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias, float* x,
                             int64_t ldx, int M, int N, int K, int rows_per_batch, const float* gate,
                             int64_t gate_batch_stride, cudaStream_t stream) {
  if (a == nullptr || w == nullptr || x == nullptr)
    return fail(ICSA_ERR_INVALID, "linear_residual: a, w and x must be non-NULL");
  if (M < 0 || N < 32 || N % 32 != 0 || K < 8 || K % 8 != 0 || rows_per_batch < 1)
    return fail(ICSA_ERR_INVALID, "linear_residual: M=%d N=%d K=%d rows_per_batch=%d (N a multiple of 32, K of 8)", M,
                N, K, rows_per_batch);
  if (lda < K || lda % 8 != 0 || ldw < K || ldw % 8 != 0 || ldx < N || ldx % 4 != 0)
    return fail(ICSA_ERR_INVALID, "linear_residual: leading dimensions (lda, ldw multiples of 8 and >= K; ldx a "
                                  "multiple of 4 and >= N)");
  if (gate != nullptr && (gate_batch_stride < 0 || gate_batch_stride % 4 != 0))
    return fail(ICSA_ERR_INVALID, "linear_residual: gate_batch_stride must be a non-negative multiple of 4");
  const void* ptrs[5] = {a, w, bias, x, gate};
  for (int i = 0; i < 5; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0)
      return fail(ICSA_ERR_INVALID, "linear_residual: buffers must be 16-byte aligned");
  if (M == 0) return ICSA_OK;
  CUtensorMap am, wm;
  int rc;
  if ((rc = encode_matrix_map(&am, a, M, K, lda)) != ICSA_OK) return rc;
  if ((rc = encode_matrix_map(&wm, w, N, K, ldw)) != ICSA_OK) return rc;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "linear_residual: device query");
  e = icsa::launch_linear_residual(M, N, K, am, wm, static_cast<const __nv_bfloat16*>(bias), x, ldx, gate,
                                   gate_batch_stride, rows_per_batch, sms, stream);
  return e == cudaSuccess ? ICSA_OK : cuda_fail(e, "linear_residual");
}

int icsa_last_status(cudaStream_t stream, int clear) {
  constexpr int kUnits = 6;
  static std::mutex mu;
  static int* addr[kMaxDevices][kUnits] = {};
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(ICSA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev][0] == nullptr) {
    cudaError_t (*const get[kUnits])(int**) = {icsa::sticky_status_dense_pair, icsa::sticky_status_flat,
                                               icsa::sticky_status_sparse, icsa::sticky_status_selftest,
                                               icsa::sticky_status_gemm, icsa::sticky_status_scores};
    int* a[kUnits] = {};
    for (int i = 0; i < kUnits; ++i)
      if ((e = get[i](&a[i])) != cudaSuccess) return cuda_fail(e, "sticky status address");
    for (int i = 0; i < kUnits; ++i) addr[dev][i] = a[i];
  }
  int first = 0;
  for (int i = 0; i < kUnits; ++i) {
    int code = 0;
    if ((e = cudaMemcpy(&code, addr[dev][i], sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
      return cuda_fail(e, "sticky status read");
    if (code != 0 && first == 0) first = code;
    if (code != 0 && clear && (e = cudaMemset(addr[dev][i], 0, sizeof(int))) != cudaSuccess)
      return cuda_fail(e, "sticky status clear");
  }
  if (first != 0)
    return fail(ICSA_ERR_DEVICE_TIMEOUT, "a device-side wait on device %d gave up since the last check (code 0x%x)",
                dev, first);
  return ICSA_OK;
}

}  // extern "C"
