// Selective-scan launch arguments shared by the forward (scan_fwd.cuh) and
// backward (scan_bwd.cuh) kernels and the finalize step, and the decoupled
// lookback helpers.
//
// Segments: when there are too few (batch row, channel tile) chains to fill
// the GPU the sequence is cut into segments that run as separate CTAs of the
// same launch, joined by flagged carries (see "segment carries").
#pragma once

#include "common.cuh"
#include "../../include/selectssm_b200.h"

namespace ssm {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------- arguments
struct FwdDir {
  CUtensorMap tm_u, tm_delta, tm_B, tm_C, tm_z;  // 64-byte aligned members first
  const float* A;
  const float* D;
  const float* bias;
  void* out;
  float* states;
  int32_t* status;
  float* segI;    // (B, nseg, D, 16) inclusive end state of each segment
  int* seg_flag;  // (B, channel tiles, nseg) lookback flags
  int64_t out_stride;
  int L, Dm, flags, gate_act, has_z;
  int nseg, seg_chunks;  // sequence segments (each seg_chunks chunks of 16 steps)
};
struct FwdLaunch {
  FwdDir dir[2];
  int zdiv;  // blockIdx.z = direction * zdiv + segment
  int* ticket;  // CTA order counter (zeroed per call); null when nothing is segmented
  int chains, ntile, batch;
  uint32_t spin_limit;
};

struct BwdDir {
  CUtensorMap tm_u, tm_delta, tm_B, tm_C, tm_z, tm_dout;  // activation boxes: 128 channels x 16 steps
  const float* states;  // (B, ceil(L/8), D, 16) forward checkpoints
  const float* A;
  const float* D;
  const float* bias;
  void* du;
  void* ddelta;
  void* dz;
  float* bc_part;  // (channel tiles, B, L, 32) per-tile dB | dC partial sums (kBcLocal)
  float* dB_acc;   // kBcMulticast: NVLink multicast addresses of the dB / dC sums (row stride acc_stride)
  float* dC_acc;
  int bc_mode;     // kBcLocal / kBcMulticast
  float* dA_part;  // (B, nseg, D, 16)
  float* dD_part;  // (B, nseg, D)
  float* db_part;  // (B, nseg, D)
  float* segI;     // (B, nseg, D, 16) adjoint carried out of each segment's first step
  int* seg_flag;   // (B, channel tiles, nseg) flags: the segment's segI is published
  int32_t* status;
  int64_t z_stride, acc_stride;
  int L, Dm, flags, gate_act, has_z;
  int nseg, seg_chunks;
};
// How the backward delivers its dB / dC partial sums (sums over a CTA's channels).
constexpr int kBcLocal = 0;      // plain stores into bc_part, summed over tiles in a fixed order by finalize
constexpr int kBcMulticast = 1;  // multimem.red at dB_acc / dC_acc (NVLink multicast addresses)

struct BwdLaunch {
  BwdDir dir[2];
  int zdiv;
  int* ticket;       // CTA order counter (zeroed per call); null when nothing is segmented
  int ticket_base;   // added to every ticket (0; the lookback self-test skips the last segment)
  int chains;        // CTAs per segment: channel tiles x batch rows x directions
  int ntile, batch;
  uint32_t spin_limit;  // polls of a lookback flag before giving up
};

// ---------------------------------------------------------------- segment carries
// Segments of one chain run their aggregate passes (the recurrence over their
// own steps from a zero start) in parallel; each then waits for the inclusive
// carry of its neighbour in scan order (flag kInclReady), composes its own and
// publishes it.  CTAs take their segment from an atomic ticket in scan order,
// so every segment a CTA waits for belongs to a CTA that is already resident
// or finished.
constexpr int kInclReady = 1;
constexpr uint32_t kLookbackSpin = 1u << 22;  // polls (each sleeps ~0.1 us): seconds, far above any real wait

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Polls *flag until it is non-zero; returns its value, or 0 after `limit` polls.
__device__ __forceinline__ int wait_flag_bounded(const int* flag, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    const int v = ld_acquire_gpu(flag);
    if (v) return v;
    __nanosleep(100);
  }
  return 0;
}
// CTA-wide wait: thread 0 polls, the result is broadcast through `slot`, and
// every thread then re-reads the flag with acquire semantics so its own later
// loads of the published values are ordered after the publisher's stores.
__device__ __forceinline__ int cta_wait_flag(const int* flag, uint32_t limit, int* slot) {
  if (threadIdx.x == 0) *slot = wait_flag_bounded(flag, limit);
  __syncthreads();
  const int v = *slot;
  __syncthreads();
  if (v) (void)ld_acquire_gpu(flag);
  return v;
}

template <typename T>
__device__ __forceinline__ void st_act(T* p, float v) {
  *p = Cvt<T>::from_f(v);
}

// Sums the per-(batch row, segment) partials of dA / dD / d(bias) in row order
// and the per-channel-tile dB / dC partials in tile order (both deterministic),
// writing dB / dC in the caller's dtype and row stride.
struct FinalizeDir {
  const float* dA_part;
  const float* dD_part;
  const float* db_part;
  float* dA;
  float* dD;
  float* dbias;
  const float* bc_part;  // (ntile, batch, L, 32) or null (dB / dC delivered elsewhere)
  void* dB;
  void* dC;
  int64_t bc_stride;
  int prows;  // rows of partials (batch x segments)
  int ntile;  // channel tiles of the backward
  int batch, L, Dm;
};

}  // namespace ssm
