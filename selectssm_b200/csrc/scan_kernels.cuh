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
  CUtensorMap tm_u, tm_delta, tm_B, tm_C, tm_z, tm_dout, tm_states;
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
    }

    if (cvalid) {
      float4* sp = reinterpret_cast<float4*>(a.states + (((size_t)b * nblk + j) * Dm + c) * kN + nq * kNL);
      *sp = make_float4(h[0], h[1], h[2], h[3]);
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

// ---------------------------------------------------------------- backward
// Compiler-only fence between unrolled steps: keeps the scheduler from
// hoisting many steps' shared-memory loads ahead of use (which costs registers).
__device__ __forceinline__ void sched_fence() { asm volatile("" ::: "memory"); }

struct BwdLane {
  int lane, nq, warp;
  bool up4, up3, up2, has_z;
};

// Reduce-scatter of 4 values over the 8 channel lanes of a warp (lane bits 2..4):
// returns the sum over the 8 channels of value k = 2*up4 + up3 (valid where !up2).
__device__ __forceinline__ float reduce_scatter4(const BwdLane& ln, float v0, float v1, float v2, float v3) {
  const float r0 = (ln.up4 ? v2 : v0) + __shfl_xor_sync(kFull, ln.up4 ? v0 : v2, 16);
  const float r1 = (ln.up4 ? v3 : v1) + __shfl_xor_sync(kFull, ln.up4 ? v1 : v3, 16);
  float q = (ln.up3 ? r1 : r0) + __shfl_xor_sync(kFull, ln.up3 ? r0 : r1, 8);
  q += __shfl_xor_sync(kFull, q, 4);
  return q;
}

// Backward shared-memory layout (bytes), sized at run time: the output-frame
// copies of u and the scan-frame copies of dout / z only exist for the reverse
// direction with the reference's skip frame.
struct BwdLayout {
  int offU, offDelta, offDo, offZo, offUo, offDs, offZs, offB, offC, offS, stage;
  int offRed, offBars, offTmem, bytes;
  __host__ __device__ BwdLayout(int es, int esbc, bool has_z, bool need_mirror) {
    const int act = kChunk * kTileCh * es, bc = kChunk * kN * esbc;
    int o = 0;
    offU = o; o += act;
    offDelta = o; o += act;
    offDo = o; o += act;
    offZo = o; if (has_z) o += act;
    offUo = o; if (need_mirror) o += act;
    offDs = o; if (need_mirror) o += act;
    offZs = o; if (need_mirror && has_z) o += act;
    offB = o; o += bc;
    offC = o; o += bc;
    offS = o; o += kTileCh * kN * 4;     // chunk-start state tile (fp32)
    stage = (o + 127) & ~127;
    offRed = stage * kBwdStages;          // two dB/dC partial buffers
    offBars = offRed + 2 * kWarps * kChunk * 32 * 4;
    offTmem = offBars + 8 * kBwdStages;
    bytes = offTmem + 16;
  }
  // bytes one stage's TMA loads deliver (the start state only when j > 0)
  __host__ __device__ uint32_t tx(int es, int esbc, bool has_z, bool need_mirror, bool with_state) const {
    const int act = kChunk * kTileCh * es, bc = kChunk * kN * esbc;
    return 3 * act + 2 * bc + (has_z ? act : 0) + (need_mirror ? (has_z ? 3 : 2) * act : 0) +
           (with_state ? kTileCh * kN * 4 : 0);
  }
};

// TMEM columns per CTA: 16 steps x (4 alpha + 4 alpha*h) per lane.
constexpr uint32_t kBwdTmemCols = kChunk * 2 * kNL;

template <typename T, typename TBC>
__global__ void __launch_bounds__(kThreads, 4) ssm_bwd_kernel(const __grid_constant__ BwdLaunch P) {
  const BwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = blockIdx.z % P.zdiv;
  extern __shared__ __align__(1024) unsigned char smem[];

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kTileCh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ch = lane >> 2, nq = lane & 3;
  const int cl = warp * kChPerWarp + ch;
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;
  const bool rev = (a.flags & SSM_REVERSE) != 0;
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool aligned = (a.flags & SSM_ALIGNED_SKIP) != 0;
  const bool softplus = (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  const bool has_z = a.has_z != 0, has_D = a.D != nullptr;
  const bool mirror = has_D && rev && !aligned;  // skip frame of the reverse direction
  const int nblk = (L + kChunk - 1) / kChunk;
  const int j1 = min(nblk, (seg + 1) * a.seg_chunks);
  const int nloc = j1 - seg * a.seg_chunks;
  const bool cvalid = c < Dm;
  const int co = comp ? Dm - 1 - c : c;
  const int oc0 = comp ? Dm - kTileCh - c0 : c0;
  const BwdLayout S(sizeof(T), sizeof(TBC), has_z, mirror);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.offBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S.offTmem);
  float* sRed = reinterpret_cast<float*>(smem + S.offRed);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kBwdTmemCols);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tbase = *tmem_slot;
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);  // this warp's lane quarter

  // it-th issue loads chunk j = j1-1-it (the segment's chunks, last first)
  auto issue = [&](int it) {
    const int j = j1 - 1 - it;
    unsigned char* st = smem + (it % kBwdStages) * S.stage;
    uint64_t* bar = &bars[it % kBwdStages];
    const int t0 = j * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, S.tx(sizeof(T), sizeof(TBC), has_z, mirror, j > 0));
    tma_load_3d(st + S.offU, &a.tm_u, bar, c0, t0, b);
    tma_load_3d(st + S.offDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S.offB, &a.tm_B, bar, 0, t0, b);
    tma_load_3d(st + S.offC, &a.tm_C, bar, 0, t0, b);
    tma_load_3d(st + S.offDo, &a.tm_dout, bar, oc0, ot0, b);
    if (has_z) tma_load_3d(st + S.offZo, &a.tm_z, bar, oc0, ot0, b);
    if (mirror) {
      tma_load_3d(st + S.offUo, &a.tm_u, bar, oc0, ot0, b);
      tma_load_3d(st + S.offDs, &a.tm_dout, bar, c0, t0, b);
      if (has_z) tma_load_3d(st + S.offZs, &a.tm_z, bar, c0, t0, b);
    }
    if (j > 0) tma_load_3d(st + S.offS, &a.tm_states, bar, 0, c0, b * nblk + j - 1);
  };
  if (threadIdx.x == 0) {
    const int npre = nloc < kBwdStages ? nloc : kBwdStages;
    for (int it = 0; it < npre; ++it) issue(it);
  }

  float An[kNL];
#pragma unroll
  for (int k = 0; k < kNL; ++k) An[k] = cvalid ? a.A[(size_t)c * kN + nq * kNL + k] : 0.f;
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsc = (has_D && cvalid) ? a.D[c] : 0.f;                         // skip weight, scan channel
  const float Dso = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;          // skip weight in pre-gate value
  float fa[kNL] = {0.f, 0.f, 0.f, 0.f};   // f_{t+1} * alpha_{t+1} carried backwards
  if (a.nseg > 1 && cvalid) {  // adjoint entering this segment from the later ones
    const float4 F = *reinterpret_cast<const float4*>(a.segF + (((size_t)b * a.nseg + seg) * Dm + c) * kN + nq * kNL);
    fa[0] = F.x; fa[1] = F.y; fa[2] = F.z; fa[3] = F.w;
  }
  float dA[kNL] = {0.f, 0.f, 0.f, 0.f};
  float dD_acc = 0.f, db_acc = 0.f;
  T* du_g = reinterpret_cast<T*>(a.du);
  T* dd_g = reinterpret_cast<T*>(a.ddelta);
  T* dz_g = reinterpret_cast<T*>(a.dz);
  const BwdLane ln{lane, nq, warp, (lane & 16) != 0, (lane & 8) != 0, (lane & 4) != 0, has_z};
  const int red_n = nq * kNL + (ln.up4 ? 2 : 0) + (ln.up3 ? 1 : 0);
  bool failed = false;

  for (int it = 0; it < nloc; ++it) {
    const int j = j1 - 1 - it;
    const int s = it % kBwdStages;
    const bool ok = mbar_wait_bounded(&bars[s], (it / kBwdStages) & 1);
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    const unsigned char* st = smem + s * S.stage;
    const T* su = reinterpret_cast<const T*>(st + S.offU);
    const T* sd = reinterpret_cast<const T*>(st + S.offDelta);
    const T* szo = reinterpret_cast<const T*>(st + S.offZo);
    const T* sdo = reinterpret_cast<const T*>(st + S.offDo);
    const T* suo = reinterpret_cast<const T*>(st + S.offUo);
    const T* szs = reinterpret_cast<const T*>(st + S.offZs);
    const T* sds = reinterpret_cast<const T*>(st + S.offDs);
    const TBC* sB = reinterpret_cast<const TBC*>(st + S.offB);
    const TBC* sC = reinterpret_cast<const TBC*>(st + S.offC);
    const float* sS = reinterpret_cast<const float*>(st + S.offS);
    float* red = sRed + (it & 1) * (kWarps * kChunk * 32);
    const int col = comp ? kTileCh - 1 - cl : cl;

    // ---- per-step scalars for the lane's 4 steps (tl = nq + 4i)
    float dtv[4], dtx[4], dys[4];
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
      const int row = rev ? kChunk - 1 - tl : tl;
      float g = ld_f(sdo + row * kTileCh + col);
      if (has_z) g *= act_f(ld_f(szo + row * kTileCh + col), a.gate_act);
      dys[i] = valid ? g : 0.f;
    }

    // ---- forward recompute from the chunk-start state; alpha_t and
    // alpha_t h_{t-1} of every step go to TMEM (columns 8 tl .. 8 tl + 7)
    float h[kNL];
    if (j > 0) {
      const float4 h0 = *reinterpret_cast<const float4*>(sS + cl * kN + nq * kNL);
      h[0] = h0.x; h[1] = h0.y; h[2] = h0.z; h[3] = h0.w;
    } else {
      h[0] = h[1] = h[2] = h[3] = 0.f;
    }
    float yv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int tl = 0; tl < kChunk; ++tl) {
      sched_fence();
      const int src = (lane & ~3) | (tl & 3);
      const float dt = __shfl_sync(kFull, dtv[tl >> 2], src);
      const float dx = __shfl_sync(kFull, dtx[tl >> 2], src);
      const float dy = __shfl_sync(kFull, dys[tl >> 2], src);
      const float dt2 = dt * kLog2e;
      const float4 Bv = ld4(sB + tl * kN + nq * kNL);
      const float4 Cv = ld4(sC + tl * kN + nq * kNL);
      const float bv[4] = {Bv.x, Bv.y, Bv.z, Bv.w};
      float keep[8];
#pragma unroll
      for (int k = 0; k < kNL; ++k) {
        const float al = ex2(An[k] * dt2);
        const float q = al * h[k];
        h[k] = fmaf(bv[k], dx, q);
        keep[k] = al;
        keep[4 + k] = q;
      }
      tmem_st8(trow + tl * 8, keep);
      if (has_z) {
        float yp = Cv.x * h[0] + Cv.y * h[1] + Cv.z * h[2] + Cv.w * h[3];
        yp += __shfl_xor_sync(kFull, yp, 1);
        yp += __shfl_xor_sync(kFull, yp, 2);
        if ((tl & 3) == nq) yv[tl >> 2] = yp;
      }
      const float sc = reduce_scatter4(ln, dy * h[0], dy * h[1], dy * h[2], dy * h[3]);
      if (!ln.up2) red[(warp * kChunk + tl) * 32 + kN + red_n] = sc;
    }
    tmem_wait_st();

    // ---- dz (needs the recomputed pre-gate output)
    if (has_z) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tl = nq + 4 * i;
        const int t = j * kChunk + tl;
        if (t < L && cvalid) {
          const int row = rev ? kChunk - 1 - tl : tl;
          const int l = rev ? L - 1 - t : t;
          float pre = yv[i];
          if (has_D) pre = fmaf(Dso, mirror ? ld_f(suo + row * kTileCh + col) : ld_f(su + tl * kTileCh + cl), pre);
          const float zz = ld_f(szo + row * kTileCh + col);
          const float g = ld_f(sdo + row * kTileCh + col) * pre * act_grad_f(zz, a.gate_act);
          st_act(dz_g + ((size_t)b * L + l) * a.z_stride + co, g);
        }
      }
    }

    // ---- adjoint sweep, steps 15..0, two steps per TMEM load
    float dxs[4], ddt[4];
    uint32_t buf[2][16];  // alternating step-pair buffers (static indices once unrolled)
    tmem_ld16(trow + (kChunk - 2) * 8, buf[(kChunk / 2 - 1) & 1]);
    tmem_wait_ld();
#pragma unroll
    for (int pr = kChunk / 2 - 1; pr >= 0; --pr) {
      if (pr > 0) tmem_ld16(trow + (2 * pr - 2) * 8, buf[(pr - 1) & 1]);
#pragma unroll
      for (int half = 1; half >= 0; --half) {
        const int tl = 2 * pr + half;
        sched_fence();
        const int src = (lane & ~3) | (tl & 3);
        const float dt = __shfl_sync(kFull, dtv[tl >> 2], src);
        const float dx = __shfl_sync(kFull, dtx[tl >> 2], src);
        const float dy = __shfl_sync(kFull, dys[tl >> 2], src);
        const float4 Bv = ld4(sB + tl * kN + nq * kNL);
        const float4 Cv = ld4(sC + tl * kN + nq * kNL);
        const float bv[4] = {Bv.x, Bv.y, Bv.z, Bv.w};
        const float cv[4] = {Cv.x, Cv.y, Cv.z, Cv.w};
        float sAw = 0.f, sBf = 0.f, vB[kNL];
#pragma unroll
        for (int k = 0; k < kNL; ++k) {
          const float al = __uint_as_float(buf[pr & 1][half * 8 + k]);
          const float q = __uint_as_float(buf[pr & 1][half * 8 + 4 + k]);
          const float f = fmaf(cv[k], dy, fa[k]);
          const float w = f * q;
          dA[k] = fmaf(dt, w, dA[k]);
          sAw = fmaf(An[k], w, sAw);
          sBf = fmaf(bv[k], f, sBf);
          vB[k] = dx * f;
          fa[k] = f * al;
        }
        sAw += __shfl_xor_sync(kFull, sAw, 1);
        sBf += __shfl_xor_sync(kFull, sBf, 1);
        sAw += __shfl_xor_sync(kFull, sAw, 2);
        sBf += __shfl_xor_sync(kFull, sBf, 2);
        if ((tl & 3) == nq) {
          dxs[tl >> 2] = dt * sBf;
          ddt[tl >> 2] = fmaf(ld_f(su + tl * kTileCh + cl), sBf, sAw);  // x sum_n B f + sum_n A w
        }
        const float sb = reduce_scatter4(ln, vB[0], vB[1], vB[2], vB[3]);
        if (!ln.up2) red[(warp * kChunk + tl) * 32 + red_n] = sb;
      }
      if (pr > 0) tmem_wait_ld();
    }

    // ---- epilogue: du, ddelta, skip grads
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tl = nq + 4 * i;
      const int t = j * kChunk + tl;
      if (t < L && cvalid) {
        const float x = ld_f(su + tl * kTileCh + cl);
        float du = dxs[i];
        if (has_D) {
          float sg = dys[i];
          if (mirror) {
            sg = ld_f(sds + tl * kTileCh + cl);
            if (has_z) sg *= act_f(ld_f(szs + tl * kTileCh + cl), a.gate_act);
          }
          du = fmaf(Dsc, sg, du);
          dD_acc = fmaf(sg, x, dD_acc);
        }
        float g = ddt[i];
        if (softplus) g *= sigmoid_f(ld_f(sd + tl * kTileCh + cl) + bias);
        db_acc += g;
        const size_t off = ((size_t)b * L + t) * Dm + c;
        st_act(du_g + off, du);
        st_act(dd_g + off, g);
      }
    }

    __syncthreads();  // stage s consumed; red[] complete
    if (threadIdx.x == 0 && it + kBwdStages < nloc) {
      fence_proxy_async_smem();
      issue(it + kBwdStages);
    }
    {
      // sum the 4 warps' partials; thread -> (step, 4 consecutive outputs)
      const int tl = threadIdx.x >> 3, q4 = threadIdx.x & 7;
      const int t = j * kChunk + tl;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float4 p = *reinterpret_cast<const float4*>(red + (w * kChunk + tl) * 32 + q4 * 4);
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      if (t < L) {
        float* dst = (q4 < 4 ? a.dB_acc : a.dC_acc) + ((size_t)b * L + t) * a.acc_stride + (q4 & 3) * 4;
        atomicAdd(reinterpret_cast<float4*>(dst), v);
      }
    }
  }

  // release TMEM (every thread's accesses are complete)
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, kBwdTmemCols);
  if (failed) {
    if (threadIdx.x == 0) report(a.status, kStatusTimeout);
    return;
  }

  // per-(batch row, segment, channel) partials of the parameter gradients
  dD_acc += __shfl_xor_sync(kFull, dD_acc, 1);
  dD_acc += __shfl_xor_sync(kFull, dD_acc, 2);
  db_acc += __shfl_xor_sync(kFull, db_acc, 1);
  db_acc += __shfl_xor_sync(kFull, db_acc, 2);
  if (cvalid) {
    const size_t r = (size_t)b * a.nseg + seg;
    *reinterpret_cast<float4*>(a.dA_part + (r * Dm + c) * kN + nq * kNL) = make_float4(dA[0], dA[1], dA[2], dA[3]);
    if (nq == 0) {
      a.dD_part[r * Dm + c] = dD_acc;
      a.db_part[r * Dm + c] = db_acc;
    }
  }
}

// Backward segment pre-pass: for segment s >= 1 runs the adjoint recurrence
// f_t = C_t dy_t + f_{t+1} alpha_{t+1} over the segment from a zero carry and
// writes the carry leaving its first step (f alpha) and the segment's sum of
// dt.  Only delta, C, dout (and z for the gate) are read.
template <typename T, typename TBC>
struct BwdAggSmem {
  static constexpr int kAct = kChunk * kTileCh * (int)sizeof(T);
  static constexpr int kBC = kChunk * kN * (int)sizeof(TBC);
  static constexpr int kOffDelta = 0, kOffDo = kAct, kOffZo = 2 * kAct, kOffC = 3 * kAct;
  static constexpr int kStage = 3 * kAct + kBC;
  static constexpr int kBars = kStage * kFwdStages;
  static constexpr int kBytes = kBars + 8 * kFwdStages;
};

template <typename T, typename TBC>
__global__ void __launch_bounds__(kThreads, 4) ssm_bwd_agg_kernel(const __grid_constant__ BwdLaunch P) {
  using S = BwdAggSmem<T, TBC>;
  const BwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = 1 + blockIdx.z % P.zdiv;  // segments 1 .. nseg-1
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kTileCh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ch = lane >> 2, nq = lane & 3;
  const int cl = warp * kChPerWarp + ch;
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;
  const bool rev = (a.flags & SSM_REVERSE) != 0;
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool softplus = (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  const bool has_z = a.has_z != 0;
  const int nblk = (L + kChunk - 1) / kChunk;
  const int j0 = seg * a.seg_chunks;
  const int j1 = min(nblk, j0 + a.seg_chunks);
  const int nloc = j1 - j0;
  const bool cvalid = c < Dm;
  const int oc0 = comp ? Dm - kTileCh - c0 : c0;
  const int col = comp ? kTileCh - 1 - cl : cl;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t tx = 2 * S::kAct + S::kBC + (has_z ? S::kAct : 0);
  auto issue = [&](int it) {
    const int j = j1 - 1 - it;
    unsigned char* st = smem + (it % kFwdStages) * S::kStage;
    uint64_t* bar = &bars[it % kFwdStages];
    const int t0 = j * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, tx);
    tma_load_3d(st + S::kOffDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S::kOffC, &a.tm_C, bar, 0, t0, b);
    tma_load_3d(st + S::kOffDo, &a.tm_dout, bar, oc0, ot0, b);
    if (has_z) tma_load_3d(st + S::kOffZo, &a.tm_z, bar, oc0, ot0, b);
  };
  if (threadIdx.x == 0) {
    const int npre = nloc < kFwdStages ? nloc : kFwdStages;
    for (int it = 0; it < npre; ++it) issue(it);
  }
  float A2[kNL];
#pragma unroll
  for (int k = 0; k < kNL; ++k) A2[k] = cvalid ? a.A[(size_t)c * kN + nq * kNL + k] * kLog2e : 0.f;
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  float fa[kNL] = {0.f, 0.f, 0.f, 0.f};
  float tsum = 0.f;
  for (int it = 0; it < nloc; ++it) {
    const int j = j1 - 1 - it;
    const int s = it % kFwdStages;
    const bool ok = mbar_wait_bounded(&bars[s], (it / kFwdStages) & 1);
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) report(a.status, kStatusTimeout);
      return;
    }
    const unsigned char* st = smem + s * S::kStage;
    const T* sd = reinterpret_cast<const T*>(st + S::kOffDelta);
    const T* sdo = reinterpret_cast<const T*>(st + S::kOffDo);
    const T* szo = reinterpret_cast<const T*>(st + S::kOffZo);
    const TBC* sC = reinterpret_cast<const TBC*>(st + S::kOffC);
    float dtv[4], dys[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tl = nq + 4 * i;
      const bool valid = j * kChunk + tl < L;
      const float dr = ld_f(sd + tl * kTileCh + cl) + bias;
      const float dt = softplus ? softplus_f(dr) : dr;
      dtv[i] = valid ? dt : 0.f;
      tsum += dtv[i];
      const int row = rev ? kChunk - 1 - tl : tl;
      float g = ld_f(sdo + row * kTileCh + col);
      if (has_z) g *= act_f(ld_f(szo + row * kTileCh + col), a.gate_act);
      dys[i] = valid ? g : 0.f;
    }
#pragma unroll
    for (int tl = kChunk - 1; tl >= 0; --tl) {
      const int src = (lane & ~3) | (tl & 3);
      const float dt = __shfl_sync(kFull, dtv[tl >> 2], src);
      const float dy = __shfl_sync(kFull, dys[tl >> 2], src);
      const float4 Cv = ld4(sC + tl * kN + nq * kNL);
      fa[0] = fmaf(Cv.x, dy, fa[0]) * ex2(A2[0] * dt);
      fa[1] = fmaf(Cv.y, dy, fa[1]) * ex2(A2[1] * dt);
      fa[2] = fmaf(Cv.z, dy, fa[2]) * ex2(A2[2] * dt);
      fa[3] = fmaf(Cv.w, dy, fa[3]) * ex2(A2[3] * dt);
    }
    __syncthreads();
    if (threadIdx.x == 0 && it + kFwdStages < nloc) {
      fence_proxy_async_smem();
      issue(it + kFwdStages);
    }
  }
  tsum += __shfl_xor_sync(kFull, tsum, 1);
  tsum += __shfl_xor_sync(kFull, tsum, 2);
  if (cvalid) {
    const size_t r = (size_t)b * a.nseg + seg;
    *reinterpret_cast<float4*>(a.segF + (r * Dm + c) * kN + nq * kNL) = make_float4(fa[0], fa[1], fa[2], fa[3]);
    if (nq == 0) a.segT[r * Dm + c] = tsum;
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
