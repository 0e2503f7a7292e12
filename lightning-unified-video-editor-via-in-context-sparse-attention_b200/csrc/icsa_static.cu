// icsa_forward_static: the whole call with its scratch memory in a file-scope
// device array instead of a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory at the point of
// the call -- a plugin host that owns every allocation and hands out none, an
// embedded runtime with a fixed memory budget and no allocator, or a
// foreign-language caller (cgo, JNI, ...) with no handle on a CUDA allocator.
// They pass only their inputs and output; the library brings the scratch.
//
// Cost and limits:
//   * the array is kIcsaStaticScratchBytes (64 MiB) of device memory.  It is
//     part of this library's device code, so every GPU that loads this part
//     of the library keeps those 64 MiB until the process exits (with the
//     default lazy module loading that happens at the first call on that GPU;
//     with CUDA_MODULE_LOADING=EAGER, when the context is created);
//   * problems whose workspace (icsa_workspace_size) exceeds that size are
//     rejected with ICSA_ERR_WORKSPACE; nothing is allocated instead;
//   * all calls share the one array and it keeps the previous call's
//     contents, so calls that overlap on the GPU (different streams, or
//     different host threads without ordering) race and corrupt each other.
//     Order them on one stream.  The only region that must start at zero,
//     the device status word, is cleared by every call;
//   * the first call on each device resolves the array's device address
//     (cudaGetSymbolAddress, which may load the module).  Make that first call
//     outside any stream capture.  The address belongs to the CUDA context:
//     it is cached with the context's unique id (cuCtxGetId), so after a
//     cudaDeviceReset() the first call in the new context resolves it again;
//   * icsa_static_device_status() reads the scratch's device status word, so
//     a device-side wait that gave up in one of these calls is reported even
//     though the caller never sees the scratch.
#include <cstdio>
#include <mutex>

#include "icsa_kernels.cuh"

namespace {

constexpr size_t kIcsaStaticScratchBytes = size_t(64) << 20;

// Device-side scratch.  In host code this name is only a handle for
// cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_icsa_static_scratch[kIcsaStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // cuCtxGetId of the context the address belongs to

// Unique id of the calling thread's current context (0 if it cannot be read).
// The driver entry points are fetched through the runtime, so the library
// does not link against libcuda.
unsigned long long current_context_id() {
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) != cudaSuccess ||
        qa != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) != cudaSuccess ||
        qb != cudaDriverEntryPointSuccess)
      return 0;
    get_current = reinterpret_cast<GetCurrentFn>(a);
    get_id = reinterpret_cast<GetIdFn>(b);
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Resolves (once per device and context, with that device current) the
// device address of the scratch array.
int icsa_static_scratch_resolve(void** out, char* msg, size_t msg_len) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    snprintf(msg, msg_len, "cudaGetDevice: %s", cudaGetErrorString(e));
    return ICSA_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, msg_len, "device ordinal %d is outside the supported range", dev);
    return ICSA_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  // a context exists once the runtime has been used on this device; before
  // that the id reads 0 and the lookup below creates the primary context
  const unsigned long long ctx = current_context_id();
  if (g_scratch_ptr[dev] == nullptr || ctx == 0 || ctx != g_scratch_ctx[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_icsa_static_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      snprintf(msg, msg_len, "cudaGetSymbolAddress of the static scratch failed: %s", cudaGetErrorString(e));
      return ICSA_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = current_context_id();
  }
  *out = g_scratch_ptr[dev];
  return ICSA_OK;
}

}  // namespace

extern "C" ICSA_API size_t icsa_static_scratch_bytes(void) { return kIcsaStaticScratchBytes; }

extern "C" ICSA_API int icsa_forward_static(const icsa_problem* p, const void* q, const void* k, const void* v,
                                            const void* alpha, void* out, cudaStream_t stream) {
  const size_t need = icsa_workspace_size(p);
  if (need == 0) return ICSA_ERR_INVALID;  // icsa_last_error() already describes the problem
  if (need > kIcsaStaticScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "icsa_forward_static: this problem needs %zu bytes of scratch but the static scratch holds %zu "
             "bytes; use icsa_forward with a caller-provided workspace",
             need, kIcsaStaticScratchBytes);
    icsa_set_last_error(buf);
    return ICSA_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  char msg[256];
  const int rc = icsa_static_scratch_resolve(&scratch, msg, sizeof(msg));
  if (rc != ICSA_OK) {
    icsa_set_last_error(msg);
    return rc;
  }
  return icsa_forward(p, q, k, v, alpha, out, scratch, kIcsaStaticScratchBytes, stream);
}

extern "C" ICSA_API int icsa_static_device_status(cudaStream_t stream) {
  void* scratch = nullptr;
  char msg[256];
  const int rc = icsa_static_scratch_resolve(&scratch, msg, sizeof(msg));
  if (rc != ICSA_OK) {
    icsa_set_last_error(msg);
    return rc;
  }
  return icsa_device_status(scratch, stream);
}
