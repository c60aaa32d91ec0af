// Selective-scan forward / backward kernels for B200 (sm_100a).
//
// Work decomposition (both kernels)
//   CTA   = one batch row b  x  32 consecutive channels  x  the whole sequence.
//   warp  = 8 channels; lane = (channel ch = lane/4, state quarter nq = lane%4)
//           and owns the 4 states n = 4*nq .. 4*nq+3 of its channel in registers.
//   time  = processed in chunks of 16 steps.  Per chunk one elected thread issues
//           TMA tile loads (32 ch x 16 steps of u / delta / z / dout, 16 x 16 of
//           B and C, the chunk-start state) into a ring of shared-memory stages
//           completed on mbarriers, so HBM reads run STAGES-1 chunks ahead.
//   Each lane computes the per-step scalars (softplus(dt), dt*x, gate) for 4 of
//   the chunk's 16 steps, and shares them with its channel's other 3 lanes by
//   warp shuffles; y = C.h is reduced over those 4 lanes by two xor-shuffles.
//
// Forward: h_t = exp(A dt_t) h_{t-1} + dt_t B_t x_t (ZOH for A, Euler for B,
//   src/selectssm/selectssm.py:74-78), y_t = C_t.h_t (:90), then the D skip
//   (:238), the reverse/complement unflip (:230-231) and the gate y*act(z)
//   (:335-338).  The state after every chunk is written to `states` (fp32).
// Backward: chunks are visited last to first.  A chunk restarts from the saved
//   state, recomputes exp(A dt) and the states of its 16 steps into registers
//   (each exponential is evaluated once), then runs the adjoint
//   f_t = alpha_{t+1} f_{t+1} + C_t dy_t backwards and forms the leaf gradients
//   of src/selectssm/ssmrecscan.py:150-161:
//     dx_t = dt_t sum_n f B_t,  dA += dt_t f alpha_t h_{t-1},  dB_t = sum_d dt_t x_t f,
//     dC_t = sum_d dy_t h_t,    ddt_t = sum_n f (A alpha_t h_{t-1} + B_t x_t).
//   dB/dC are reduced over the warp's 8 channels by a shuffle reduce-scatter,
//   over the CTA's 4 warps in shared memory, and over channel tiles with one
//   16-byte atomic add per thread per chunk.  dA/dD/d(delta_bias) are written
//   as per-batch-row partials and summed in a fixed order by a finalize kernel.
#pragma once

#include "common.cuh"
#include "../../include/selectssm_b200.h"

namespace ssm {

constexpr int kFwdStages = 4;
constexpr int kBwdStages = 3;
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
  float* dB_acc;   // fp32 accumulation target for dB (row stride acc_stride)
  float* dC_acc;
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
struct BwdLaunch {
  BwdDir dir[2];
  int zdiv;
};

template <typename T>
__device__ __forceinline__ void st_act(T* p, float v) {
  *p = Cvt<T>::from_f(v);
}

// ---------------------------------------------------------------- forward
template <typename T, typename TBC>
struct FwdSmem {
  static constexpr int kAct = kChunk * kTileCh * (int)sizeof(T);   // one 16x32 activation tile
  static constexpr int kBC = kChunk * kN * (int)sizeof(TBC);        // one 16x16 B or C tile
  static constexpr int kOffU = 0, kOffDelta = kAct, kOffZ = 2 * kAct, kOffUo = 3 * kAct;
  static constexpr int kOffB = 4 * kAct, kOffC = 4 * kAct + kBC;
  static constexpr int kStage = 4 * kAct + 2 * kBC;
  static constexpr int kBars = kStage * kFwdStages;
  static constexpr int kBytes = kBars + 8 * kFwdStages;
};

// AGG: the segment pre-pass.  It runs the recurrence over one segment from a
// zero state and writes only the segment's end state and sum of dt (no C, z,
// output or checkpoints); the main pass then starts segment s from the states
// of segments 0..s-1 folded together (h <- exp(A sum dt) h + H).
template <typename T, typename TBC, bool AGG>
__global__ void __launch_bounds__(kThreads, 3) ssm_fwd_kernel(const __grid_constant__ FwdLaunch P) {
  using S = FwdSmem<T, TBC>;
  const FwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = blockIdx.z % P.zdiv;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kTileCh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ch = lane >> 2, nq = lane & 3;
  const int cl = warp * kChPerWarp + ch;
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;  // grid is sized for the larger direction
  const bool rev = (a.flags & SSM_REVERSE) != 0;
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool aligned = (a.flags & SSM_ALIGNED_SKIP) != 0;
  const bool softplus = (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  const bool has_z = a.has_z != 0, has_D = a.D != nullptr;
  const bool need_uo = has_D && rev && !aligned;
  const int nblk = (L + kChunk - 1) / kChunk;
  const int nck = (L + kCk - 1) / kCk;
  const int j0 = seg * a.seg_chunks;
  const int j1 = min(nblk, j0 + a.seg_chunks);
  const int nloc = j1 - j0;
  const bool cvalid = c < Dm;
  const int co = comp ? Dm - 1 - c : c;                 // output-frame channel
  const int oc0 = comp ? Dm - kTileCh - c0 : c0;        // output-frame tile start

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const uint32_t tx = AGG ? 2 * S::kAct + S::kBC
                          : 2 * S::kAct + 2 * S::kBC + (has_z ? S::kAct : 0) + (need_uo ? S::kAct : 0);
  auto issue = [&](int jl) {  // local chunk index within the segment
    unsigned char* st = smem + (jl % kFwdStages) * S::kStage;
    uint64_t* bar = &bars[jl % kFwdStages];
    const int t0 = (j0 + jl) * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, tx);
    tma_load_3d(st + S::kOffU, &a.tm_u, bar, c0, t0, b);
    tma_load_3d(st + S::kOffDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S::kOffB, &a.tm_B, bar, 0, t0, b);
    if (!AGG) {
      tma_load_3d(st + S::kOffC, &a.tm_C, bar, 0, t0, b);
      if (has_z) tma_load_3d(st + S::kOffZ, &a.tm_z, bar, oc0, ot0, b);
      if (need_uo) tma_load_3d(st + S::kOffUo, &a.tm_u, bar, oc0, ot0, b);
    }
  };
  if (threadIdx.x == 0) {
    const int npre = nloc < kFwdStages ? nloc : kFwdStages;
    for (int jl = 0; jl < npre; ++jl) issue(jl);
  }

  // per-lane constants
  float A2[kNL];
#pragma unroll
  for (int k = 0; k < kNL; ++k) A2[k] = cvalid ? a.A[(size_t)c * kN + nq * kNL + k] * kLog2e : 0.f;
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsk = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;
  float h[kNL] = {0.f, 0.f, 0.f, 0.f};
  if (!AGG && cvalid) {  // fold the states of the preceding segments
    for (int sp = 0; sp < seg; ++sp) {
      const size_t r = (size_t)b * a.nseg + sp;
      const float T = a.segT[r * Dm + c];
      const float4 H = *reinterpret_cast<const float4*>(a.segH + (r * Dm + c) * kN + nq * kNL);
      h[0] = fmaf(ex2(A2[0] * T), h[0], H.x);
      h[1] = fmaf(ex2(A2[1] * T), h[1], H.y);
      h[2] = fmaf(ex2(A2[2] * T), h[2], H.z);
      h[3] = fmaf(ex2(A2[3] * T), h[3], H.w);
    }
  }
  float tsum = 0.f;  // AGG: sum of this lane's dt
  T* out = reinterpret_cast<T*>(a.out);

  for (int j = j0; j < j1; ++j) {
    const int jl = j - j0;
    const int s = jl % kFwdStages;
    const bool ok = mbar_wait_bounded(&bars[s], (jl / kFwdStages) & 1);
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) report(a.status, kStatusTimeout);
      return;
    }
    const unsigned char* st = smem + s * S::kStage;
    const T* su = reinterpret_cast<const T*>(st + S::kOffU);
    const T* sd = reinterpret_cast<const T*>(st + S::kOffDelta);
    const T* sz = reinterpret_cast<const T*>(st + S::kOffZ);
    const T* suo = reinterpret_cast<const T*>(st + S::kOffUo);
    const TBC* sB = reinterpret_cast<const TBC*>(st + S::kOffB);
    const TBC* sC = reinterpret_cast<const TBC*>(st + S::kOffC);

    // per-step scalars for this lane's 4 steps (tl = nq + 4i)
    float dtv[4], dtx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tl = nq + 4 * i;
      const bool valid = j * kChunk + tl < L;
      const float x = ld_f(su + tl * kTileCh + cl);
      const float dr = ld_f(sd + tl * kTileCh + cl) + bias;
      float dt = softplus ? softplus_f(dr) : dr;
      dt = valid ? dt : 0.f;
      dtv[i] = dt;
      dtx[i] = valid ? dt * x : 0.f;
      tsum += dt;
    }
    if (AGG) {
#pragma unroll
      for (int tl = 0; tl < kChunk; ++tl) {
        const int src = (lane & ~3) | (tl & 3);
        const float dt = __shfl_sync(kFull, dtv[tl >> 2], src);
        const float dx = __shfl_sync(kFull, dtx[tl >> 2], src);
        const float4 Bv = ld4(sB + tl * kN + nq * kNL);
        h[0] = fmaf(ex2(A2[0] * dt), h[0], Bv.x * dx);
        h[1] = fmaf(ex2(A2[1] * dt), h[1], Bv.y * dx);
        h[2] = fmaf(ex2(A2[2] * dt), h[2], Bv.z * dx);
        h[3] = fmaf(ex2(A2[3] * dt), h[3], Bv.w * dx);
      }
      __syncthreads();
      if (threadIdx.x == 0 && jl + kFwdStages < nloc) {
        fence_proxy_async_smem();
        issue(jl + kFwdStages);
      }
      continue;
    }

    float yv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int tl = 0; tl < kChunk; ++tl) {
      const int src = (lane & ~3) | (tl & 3);
      const float dt = __shfl_sync(kFull, dtv[tl >> 2], src);
      const float dx = __shfl_sync(kFull, dtx[tl >> 2], src);
      const float4 Bv = ld4(sB + tl * kN + nq * kNL);
      const float4 Cv = ld4(sC + tl * kN + nq * kNL);
      h[0] = fmaf(ex2(A2[0] * dt), h[0], Bv.x * dx);
      h[1] = fmaf(ex2(A2[1] * dt), h[1], Bv.y * dx);
      h[2] = fmaf(ex2(A2[2] * dt), h[2], Bv.z * dx);
      h[3] = fmaf(ex2(A2[3] * dt), h[3], Bv.w * dx);
      float yp = Cv.x * h[0] + Cv.y * h[1] + Cv.z * h[2] + Cv.w * h[3];
      yp += __shfl_xor_sync(kFull, yp, 1);
      yp += __shfl_xor_sync(kFull, yp, 2);
      if ((tl & 3) == nq) yv[tl >> 2] = yp;
      if ((tl & (kCk - 1)) == kCk - 1) {  // checkpoint after every kCk steps
        const int ck = j * (kChunk / kCk) + tl / kCk;
        if (cvalid && ck < nck) {
          float4* sp = reinterpret_cast<float4*>(a.states + (((size_t)b * nck + ck) * Dm + c) * kN + nq * kNL);
          *sp = make_float4(h[0], h[1], h[2], h[3]);
        }
      }
    }

    // epilogue: skip, gate, store (lane's own 4 steps)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tl = nq + 4 * i;
      const int t = j * kChunk + tl;
      if (t < L && cvalid) {
        const int row = rev ? kChunk - 1 - tl : tl;
        const int col = comp ? kTileCh - 1 - cl : cl;
        const int l = rev ? L - 1 - t : t;
        float y = yv[i];
        if (has_D) {
          const float xs = need_uo ? ld_f(suo + row * kTileCh + col) : ld_f(su + tl * kTileCh + cl);
          y = fmaf(Dsk, xs, y);
        }
        if (has_z) y *= act_f(ld_f(sz + row * kTileCh + col), a.gate_act);
        st_act(out + ((size_t)b * L + l) * a.out_stride + co, y);
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (threadIdx.x == 0 && jl + kFwdStages < nloc) {
      fence_proxy_async_smem();
      issue(jl + kFwdStages);
    }
  }
  if (AGG) {
    tsum += __shfl_xor_sync(kFull, tsum, 1);
    tsum += __shfl_xor_sync(kFull, tsum, 2);
    if (cvalid) {
      const size_t r = (size_t)b * a.nseg + seg;
      *reinterpret_cast<float4*>(a.segH + (r * Dm + c) * kN + nq * kNL) = make_float4(h[0], h[1], h[2], h[3]);
      if (nq == 0) a.segT[r * Dm + c] = tsum;
    }
  }
}

// Turns the per-segment adjoint aggregates into the adjoint entering each
// segment from the right, in place: carry_{S-1} = 0,
// carry_s = exp(A T_{s+1}) carry_{s+1} + F_{s+1}.  One thread per (b, d, n).
// Grid: (channel*state blocks, direction, batch row).
__global__ void ssm_bwd_fold_kernel(const __grid_constant__ BwdLaunch P) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const BwdDir& a = P.dir[blockIdx.y];
  if (i >= (int64_t)a.Dm * kN) return;
  const int b = blockIdx.z;
  const int c = (int)(i / kN), n = (int)(i % kN);
  const float A2 = a.A[(size_t)c * kN + n] * kLog2e;
  float carry = 0.f;
  for (int sg = a.nseg - 1; sg >= 0; --sg) {
    const size_t r = (size_t)b * a.nseg + sg;
    float* Fp = a.segF + (r * a.Dm + c) * kN + n;
    const float F = sg > 0 ? *Fp : 0.f;
    const float T = sg > 0 ? a.segT[r * a.Dm + c] : 0.f;
    *Fp = carry;
    carry = fmaf(ex2(A2 * T), carry, F);
  }
}

// Sums the per-batch-row partials in batch order (deterministic) and converts
// the fp32 dB/dC accumulators when B/C are bf16.
struct FinalizeDir {
  const float* dA_part;
  const float* dD_part;
  const float* db_part;
  float* dA;
  float* dD;
  float* dbias;
  const float* dB_acc;
  const float* dC_acc;
  void* dB;
  void* dC;
  int64_t bc_stride;
  int prows;  // rows of partials (batch x segments)
  int batch, L, Dm, convert_bc;
};

}  // namespace ssm
