// Self-test of the kernels' failure path: a bounded mbarrier wait that can
// never complete (nothing arrives on the barrier) must give up after its poll
// limit, record SSM_ERR_TIMEOUT in the status word and return, leaving the
// context usable.  It runs the same wait helper the scan kernels use, so a
// caller (or a test) can check the path without provoking a real fault.

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "../../include/selectssm_b200.h"

namespace ssm {

int launch_error(const char* where, cudaError_t e);  // scan.cu
int bind_device(const void* ptr);                      // scan.cu

__global__ void selftest_wait_kernel(int32_t* status, uint32_t spin_limit) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait_bounded(&bar, 0, spin_limit);
  if (!__syncthreads_and(ok) && threadIdx.x == 0) report(status, kStatusTimeout);
}

}  // namespace ssm

using namespace ssm;

extern "C" int ssm_selftest_wait_timeout(int32_t* status, uint32_t spin_limit, ssm_stream_t stream) {
  if (!status) return SSM_ERR_NULL;
  if (spin_limit == 0 || spin_limit > kSpinLimit) return SSM_ERR_SHAPE;
  int st = bind_device(status);
  if (st) return st;
  selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status, spin_limit);
  note_launches(1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SSM_OK : launch_error("launch selftest_wait_kernel", e);
}
