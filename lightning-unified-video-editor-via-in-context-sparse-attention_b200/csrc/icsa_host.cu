// icsa_forward_host: the whole call for q, k, v and output in HOST memory,
// streamed through the GPU by groups of heads.
//
// Every stage of the call is independent per (batch, head), so the heads are
// processed in groups of `group_heads`.  Each group goes through three
// streams, overlapping one group's copy to the device with another group's
// computation and a third group's copy back:
//
//   copy-in stream   H2D of the group's q, k, v columns
//   caller's stream  icsa_forward on the group (H = group_heads)
//   copy-out stream  D2H of the group's output columns
//
// The copy to the device is the slowest stream, so what remains after it is
// the computation and copy back of the last group; the last full group is
// therefore split into smaller groups (5 -> 3, 1, 1) to shorten that tail.
//
// A group of heads is a strided slice of the [B, S, H, D] host buffers: rows
// of group_heads * D elements, H * D elements apart.  cudaMemcpy2DAsync copies
// it to / from a compact [B, S, group_heads, D] device buffer.  Three buffer
// slots rotate, so a slot is refilled only after the copy-out of the group it
// last held.  The calling thread returns after enqueueing; the caller's
// stream completes when the last output column has reached host memory.
// Host buffers should be pinned (page-locked); pageable memory works but
// makes the copies synchronous.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "icsa_kernels.cuh"

extern "C" void icsa_set_last_error(const char* msg);

namespace {

constexpr int kSlots = 3;
constexpr int kMaxDevices = 64;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
size_t elem_size(int dt) { return dt == ICSA_F32 ? 4 : 2; }

int host_fail(int code, const char* msg) {
  icsa_set_last_error(msg);
  return code;
}

int host_cuda_fail(cudaError_t e, const char* where) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", where, cudaGetErrorString(e));
  icsa_set_last_error(buf);
  return ICSA_ERR_CUDA;
}

struct HostPlan {
  icsa_problem g;  // the per-group problem (H = group_heads)
  int groups;
  size_t in_bytes[3];  // compact device q, k, v of one group
  size_t out_bytes;
  size_t ws_bytes;     // icsa workspace of one group
  size_t slot_bytes;
  size_t total;        // 256 B status word + kSlots slots
};

int make_plan(const icsa_problem* p, int group_heads, HostPlan* pl) {
  if (p == nullptr) return host_fail(ICSA_ERR_INVALID, "problem is NULL");
  if (group_heads < 1 || group_heads > p->H || p->H % group_heads != 0)
    return host_fail(ICSA_ERR_INVALID, "group_heads must divide H");
  pl->g = *p;
  pl->g.H = group_heads;
  pl->groups = p->H / group_heads;
  const size_t rows = size_t(p->B) * size_t(p->S) * size_t(group_heads) * size_t(p->D);
  pl->in_bytes[0] = rows * elem_size(p->q_dtype);
  pl->in_bytes[1] = rows * elem_size(p->k_dtype);
  pl->in_bytes[2] = rows * elem_size(p->v_dtype);
  pl->out_bytes = rows * elem_size(p->out_dtype);
  pl->ws_bytes = icsa_workspace_size(&pl->g);
  if (pl->ws_bytes == 0) return ICSA_ERR_INVALID;  // icsa_workspace_size set the message
  pl->slot_bytes = align256(pl->in_bytes[0]) + align256(pl->in_bytes[1]) + align256(pl->in_bytes[2]) +
                   align256(pl->out_bytes) + align256(pl->ws_bytes);
  pl->total = 256 + size_t(kSlots) * pl->slot_bytes;
  return ICSA_OK;
}

// Per-device copy streams and slot events, created on first use.
struct DevStreams {
  bool ready = false;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t entry = nullptr;
  cudaEvent_t in_done[kSlots] = {}, comp_done[kSlots] = {}, out_done[kSlots] = {};
};
std::mutex g_host_mutex;
DevStreams g_dev[kMaxDevices];

int dev_streams(DevStreams** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return host_cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return host_fail(ICSA_ERR_UNSUPPORTED, "device ordinal out of range");
  DevStreams& d = g_dev[dev];
  if (!d.ready) {
    if ((e = cudaStreamCreateWithFlags(&d.in, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&d.out, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&d.entry, cudaEventDisableTiming)) != cudaSuccess)
      return host_cuda_fail(e, "stream / event creation");
    for (int s = 0; s < kSlots; ++s) {
      if ((e = cudaEventCreateWithFlags(&d.in_done[s], cudaEventDisableTiming)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&d.comp_done[s], cudaEventDisableTiming)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&d.out_done[s], cudaEventDisableTiming)) != cudaSuccess)
        return host_cuda_fail(e, "event creation");
    }
    d.ready = true;
  }
  *out = &d;
  return ICSA_OK;
}

// Folds a group's device status word into the call's status word (first
// nonzero code wins), so that icsa_device_status(workspace) reports a failure
// of any group.
__global__ void status_fold_kernel(int* dst, const int* src) {
  const int code = *src;
  if (code != 0) atomicCAS(dst, 0, code);
}

}  // namespace

extern "C" {

ICSA_API size_t icsa_host_workspace_size(const icsa_problem* p, int group_heads) {
  HostPlan pl;
  return make_plan(p, group_heads, &pl) == ICSA_OK ? pl.total : 0;
}

ICSA_API int icsa_forward_host(const icsa_problem* p, int group_heads, const void* q, const void* k, const void* v,
                               const void* alpha, void* out, void* workspace, size_t workspace_bytes,
                               cudaStream_t stream) {
  HostPlan pl;
  int rc = make_plan(p, group_heads, &pl);
  if (rc != ICSA_OK) return rc;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return host_fail(ICSA_ERR_INVALID, "q, k, v and out must be non-NULL");
  if (p->alpha_mode == ICSA_ALPHA_TENSOR && alpha == nullptr)
    return host_fail(ICSA_ERR_INVALID, "alpha tensor is NULL");
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return host_fail(ICSA_ERR_INVALID, "workspace must be non-NULL and 256-byte aligned");
  if (workspace_bytes < pl.total) return host_fail(ICSA_ERR_WORKSPACE, "workspace smaller than icsa_host_workspace_size()");

  std::lock_guard<std::mutex> lock(g_host_mutex);
  DevStreams* d = nullptr;
  if ((rc = dev_streams(&d)) != ICSA_OK) return rc;

  uint8_t* base = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(base);
  cudaError_t e = cudaMemsetAsync(status, 0, 256, stream);
  if (e != cudaSuccess) return host_cuda_fail(e, "status reset");
  // the copies may not start before earlier work on the caller's stream
  if ((e = cudaEventRecord(d->entry, stream)) != cudaSuccess) return host_cuda_fail(e, "event record");
  if ((e = cudaStreamWaitEvent(d->in, d->entry, 0)) != cudaSuccess) return host_cuda_fail(e, "stream wait");
  if ((e = cudaStreamWaitEvent(d->out, d->entry, 0)) != cudaSuccess) return host_cuda_fail(e, "stream wait");

  const size_t rows = size_t(p->B) * size_t(p->S);
  const void* src[3] = {q, k, v};
  const int dts[3] = {p->q_dtype, p->k_dtype, p->v_dtype};
  const size_t eo = elem_size(p->out_dtype);

  // group schedule: full groups, then the last full group in halving pieces
  // (every piece is at most group_heads, the size the slots are laid out for)
  std::vector<int> starts, sizes;
  {
    int h = 0;
    for (int g = 0; g + 1 < pl.groups; ++g, h += group_heads) {
      starts.push_back(h);
      sizes.push_back(group_heads);
    }
    for (int rest = p->H - h; rest > 0;) {
      const int piece = rest > 1 ? (rest + 1) / 2 : 1;
      starts.push_back(h);
      sizes.push_back(piece);
      h += piece;
      rest -= piece;
    }
  }
  const int ng = int(sizes.size());

  for (int g = 0; g < ng; ++g) {
    const int s = g % kSlots;
    const int hg = sizes[g];
    icsa_problem pg = pl.g;
    pg.H = hg;
    const size_t ws_g = icsa_workspace_size(&pg);
    if (ws_g == 0 || ws_g > pl.ws_bytes) return host_fail(ICSA_ERR_INVALID, "group workspace");
    uint8_t* slot = base + 256 + size_t(s) * pl.slot_bytes;
    uint8_t* dev_in[3];
    size_t off = 0;
    for (int i = 0; i < 3; ++i) {
      dev_in[i] = slot + off;
      off += align256(pl.in_bytes[i]);
    }
    uint8_t* dev_out = slot + off;
    off += align256(pl.out_bytes);
    uint8_t* ws = slot + off;
    const size_t h0 = size_t(starts[g]);
    const size_t cols = size_t(hg) * size_t(p->D);  // elements per row of this group

    // copy in (after the copy-out of the group this slot held before)
    if (g >= kSlots && (e = cudaStreamWaitEvent(d->in, d->out_done[s], 0)) != cudaSuccess)
      return host_cuda_fail(e, "stream wait");
    for (int i = 0; i < 3; ++i) {
      const size_t es = elem_size(dts[i]);
      e = cudaMemcpy2DAsync(dev_in[i], cols * es, static_cast<const uint8_t*>(src[i]) + h0 * p->D * es,
                            size_t(p->H) * p->D * es, cols * es, rows, cudaMemcpyHostToDevice, d->in);
      if (e != cudaSuccess) return host_cuda_fail(e, "copy to device");
    }
    if ((e = cudaEventRecord(d->in_done[s], d->in)) != cudaSuccess) return host_cuda_fail(e, "event record");

    // compute on the caller's stream
    if ((e = cudaStreamWaitEvent(stream, d->in_done[s], 0)) != cudaSuccess) return host_cuda_fail(e, "stream wait");
    const void* alpha_g = alpha;
    if (p->alpha_mode == ICSA_ALPHA_TENSOR && alpha != nullptr)
      alpha_g = static_cast<const uint8_t*>(alpha) +
                size_t(p->alpha_strides[2]) * h0 * elem_size(p->alpha_dtype);
    rc = icsa_forward(&pg, dev_in[0], dev_in[1], dev_in[2], alpha_g, dev_out, ws, ws_g, stream);
    if (rc != ICSA_OK) return rc;
    status_fold_kernel<<<1, 1, 0, stream>>>(status, reinterpret_cast<const int*>(ws));
    if ((e = cudaGetLastError()) != cudaSuccess) return host_cuda_fail(e, "status fold");
    if ((e = cudaEventRecord(d->comp_done[s], stream)) != cudaSuccess) return host_cuda_fail(e, "event record");

    // copy out
    if ((e = cudaStreamWaitEvent(d->out, d->comp_done[s], 0)) != cudaSuccess) return host_cuda_fail(e, "stream wait");
    e = cudaMemcpy2DAsync(static_cast<uint8_t*>(out) + h0 * p->D * eo, size_t(p->H) * p->D * eo, dev_out, cols * eo,
                          cols * eo, rows, cudaMemcpyDeviceToHost, d->out);
    if (e != cudaSuccess) return host_cuda_fail(e, "copy to host");
    if ((e = cudaEventRecord(d->out_done[s], d->out)) != cudaSuccess) return host_cuda_fail(e, "event record");
  }
  // the caller's stream completes when every output column is in host memory
  for (int s = 0; s < kSlots && s < ng; ++s)
    if ((e = cudaStreamWaitEvent(stream, d->out_done[s], 0)) != cudaSuccess) return host_cuda_fail(e, "stream wait");
  return ICSA_OK;
}

}  // extern "C"
