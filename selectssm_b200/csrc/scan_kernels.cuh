// Selective-scan launch arguments shared by the forward (scan_fwd.cuh) and
// backward (scan_bwd.cuh) kernels, the backward segment fold and the
// finalize step.
//
// Segments: when there are too few (batch row, channel tile) chains to fill
// the GPU the sequence is cut into segments that run as separate CTAs.  A
// pre-pass computes each segment's end state (forward) or the adjoint carried
// out of its first step (backward) from a zero start, plus its sum of dt; the
// main pass folds those of the neighbouring segments into its start state.
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
  float* segH;    // (B, nseg, D, 16) segment end states from a zero start
  float* segT;    // (B, nseg, D) sum of dt over each segment
  int64_t out_stride;
  int L, Dm, flags, gate_act, has_z;
  int nseg, seg_chunks;  // sequence segments (each seg_chunks chunks of 16 steps)
};
struct FwdLaunch {
  FwdDir dir[2];
  int zdiv;  // blockIdx.z = direction * zdiv + segment
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
  float* segF;     // (B, nseg, D, 16) adjoint carried out of each segment's first step, zero start
  float* segT;     // (B, nseg, D) sum of dt over each segment
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
};

template <typename T>
__device__ __forceinline__ void st_act(T* p, float v) {
  *p = Cvt<T>::from_f(v);
}

// Turns the per-segment adjoint aggregates into the adjoint entering each
// segment from the right, in place: carry_{S-1} = 0,
// carry_s = exp(A T_{s+1}) carry_{s+1} + F_{s+1}.  One thread per (b, d, n).
// The loads of a batch of 8 segments are issued before the dependent chain
// runs through them, so the chain waits on one load latency per batch.
// Grid: (channel*state blocks, direction, batch row).
__global__ void ssm_bwd_fold_kernel(const __grid_constant__ BwdLaunch P) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const BwdDir& a = P.dir[blockIdx.y];
  if (i >= (int64_t)a.Dm * kN) return;
  const int b = blockIdx.z;
  const int c = (int)(i / kN), n = (int)(i % kN);
  const float A2 = a.A[(size_t)c * kN + n] * kLog2e;
  const size_t row0 = (size_t)b * a.nseg;
  float carry = 0.f;
  constexpr int kBatch = 8;
  for (int top = a.nseg - 1; top >= 0; top -= kBatch) {
    float F[kBatch], T[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int sg = top - k;
      const size_t r = row0 + (sg > 0 ? sg : 0);
      F[k] = sg > 0 ? a.segF[(r * a.Dm + c) * kN + n] : 0.f;
      T[k] = sg > 0 ? a.segT[r * a.Dm + c] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int sg = top - k;
      if (sg >= 0) {
        a.segF[((row0 + sg) * a.Dm + c) * kN + n] = carry;
        carry = fmaf(ex2(A2 * T[k]), carry, F[k]);
      }
    }
  }
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
