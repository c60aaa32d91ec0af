// Backward scan for callers that cannot allocate device memory.
//
// Some callers of this library can't call cudaMalloc at the point where they
// run the backward: code running inside a framework whose allocator owns all
// device memory (an XLA custom call without a scratch buffer, a pre-planned
// static memory arena), or real-time callers that forbid allocation on the
// hot path.  ssm_bwd_noalloc gives them the backward of ssm_bwd with its
// scratch taken from a fixed file-scope device array instead of a caller
// workspace.  It has no counterpart in the reference.
#include <cstdio>
#include <mutex>

#include "../../include/selectssm_b200.h"
#include "common.cuh"

namespace ssm {
int bind_device(const void* ptr);                   // scan.cu
int launch_error(const char* where, cudaError_t e);  // scan.cu

// Scratch shared by every call on a device; each GPU that loads the library
// keeps it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SSM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_scratch_addr[kMaxDevices];  // device address of g_noalloc_scratch per device
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device, resolved once per
// device (the host-side name of the array is not a device address).
static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return launch_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return launch_error("device ordinal out of range", cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return launch_error("cudaGetSymbolAddress(g_noalloc_scratch)", e);
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SSM_OK;
}

}  // namespace ssm

extern "C" SSM_API int ssm_bwd_noalloc(const ssm_params_t* p, ssm_stream_t stream) {
  using namespace ssm;
  if (!p) return SSM_ERR_NULL;
  const size_t need = ssm_bwd_workspace_bytes(p, 0);
  if (need > SSM_NOALLOC_SCRATCH_BYTES) return SSM_ERR_WORKSPACE;
  const bool empty = (int64_t)p->batch * p->seqlen * p->dim == 0;
  if (!empty || p->dA) {
    const int st = bind_device(empty ? (const void*)p->dA : p->u);
    if (st) return st;
  }
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st) return st;
  ssm_params_t q = *p;
  q.workspace = scratch;
  q.workspace_bytes = SSM_NOALLOC_SCRATCH_BYTES;
  return ssm_bwd(&q, stream);
}
