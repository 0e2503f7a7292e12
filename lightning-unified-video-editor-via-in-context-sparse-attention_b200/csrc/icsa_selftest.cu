// icsa_wait_selftest: exercises the device-side bounded wait that every
// kernel of the library uses (mbar_wait), on an mbarrier that nothing ever
// arrives at.  After about one second the wait gives up, records
// kErrSelfTest in the workspace status word and the kernel returns normally,
// so the CUDA context stays usable; icsa_device_status() then reports
// ICSA_ERR_DEVICE_TIMEOUT.  No fault, trap or hang is involved.
#include "icsa_kernels.cuh"

extern "C" void icsa_set_last_error(const char* msg);

namespace {
using namespace icsa;

constexpr int kErrSelfTest = 0x1FF;

__global__ void wait_selftest_kernel(int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, status, kErrSelfTest, &abort_flag);
}

}  // namespace

namespace icsa {
ICSA_DEFINE_STICKY_ACCESSOR(sticky_status_selftest)
}  // namespace icsa

extern "C" ICSA_API int icsa_wait_selftest(void* workspace, cudaStream_t stream) {
  if (workspace == nullptr) {
    icsa_set_last_error("workspace is NULL");
    return ICSA_ERR_INVALID;
  }
  cudaError_t e = cudaMemsetAsync(workspace, 0, 256, stream);
  if (e == cudaSuccess) {
    wait_selftest_kernel<<<1, 32, 0, stream>>>(static_cast<int*>(workspace));
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    icsa_set_last_error(cudaGetErrorString(e));
    return ICSA_ERR_CUDA;
  }
  return ICSA_OK;
}
