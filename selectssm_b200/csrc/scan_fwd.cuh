// Selective-scan forward kernel for B200 (sm_100a).
//
// Work decomposition
//   CTA   = one batch row b x 32 consecutive channels x one sequence segment;
//           4 warps of 8 channels.  A channel belongs to 4 lanes
//           (lane = 4 ch + nq), each owning 4 of the 16 states
//           (n = 4 nq .. 4 nq + 3) as 2 packed f32x2 pairs.
//   time  = TMA stages of 16 steps (u, delta, z tiles of 32 ch x 16 steps, the
//           B and C tiles of 16 steps x 16 states) in a ring of shared-memory
//           stages completed on mbarriers, issued STAGES-1 stages ahead.
//   Per stage, each lane evaluates the per-step scalars softplus(dt + bias) and
//   dt x for 4 of the 16 steps (t = 4 i + nq) and the quad swaps them with
//   shuffles.  y_t = C_t . h_t is a quarter on each lane; every 4 steps a
//   reduce-scatter over the quad (3 shuffles) leaves step 4 i + nq's total on
//   lane nq, which runs that step's epilogue (D skip, gate, store).  The gate
//   activation is dispatched once per stage, so the step loops hold no branch.
//   Four lanes per channel give 4x the warps of a lane-per-channel layout,
//   enough to fill the GPU at batch 8 without cutting the sequence.
//
// Recurrence (src/selectssm/selectssm.py:74-78, :90): h_t = exp(A dt_t) h_{t-1}
// + dt_t B_t x_t, y_t = C_t . h_t; then the D skip (:238), the reverse /
// complement unflip (:230-231) and the gate y * act(z) (:335-338).  The state
// after every 8 steps is written to `states` for the backward.
//
// Segments (SEG launches): a CTA takes its segment from an atomic ticket in
// scan order; a segment that a later one depends on first runs the recurrence
// over its own steps from a zero state (the aggregate pass: u, delta, B only),
// keeping the end state H and its sum of dt T in registers, then waits
// (bounded) for the inclusive end state of the segment before it, publishes
// its own (H + exp(A T) carry) under a flag and runs the main pass from the
// true state.  Only that short step is chained, in segment order.
#pragma once

#include <type_traits>

#include "scan_kernels.cuh"

namespace ssm {



constexpr int kFThreads = 4 * kTileCh;  // 4 lanes per channel, 8 channels per warp
#ifndef SSM_FWD_MINB
#define SSM_FWD_MINB 6
#endif
constexpr int kFMinBlocks = SSM_FWD_MINB * 128 / kFThreads;  // resident CTAs per SM (80 registers at 6)
constexpr int kFStages = 3;

template <typename T, typename TBC>
struct FwdSmem {
  static constexpr int kAct = kChunk * kTileCh * (int)sizeof(T);
  static constexpr int kBC = kChunk * kN * (int)sizeof(TBC);
  static constexpr int kOffU = 0, kOffDelta = kAct, kOffZ = 2 * kAct, kOffUo = 3 * kAct;
  static constexpr int kOffB = 4 * kAct, kOffC = 4 * kAct + kBC;
  static constexpr int kStage = 4 * kAct + 2 * kBC;
  static constexpr int kBars = kStage * kFStages;  // full[kFStages] then empty[kFStages]
  static constexpr int kBytes = kBars + 16 * kFStages + 16;  // + ticket / flag broadcast words
};


// WIDE: the grid fills at most half the resident CTAs, so each thread may use
// up to twice the registers (more scheduling freedom).
// SEG: the launch cuts the sequence into segments (lookback code compiled in).
// FR: 1 (2) = a single-direction forward-frame (reverse-frame) launch with
// softplus(dt), a length of whole 16-step chunks and whole channel tiles:
// frame, softplus and bounds masks are compile-time constants; 0 = generic.
template <typename T, typename TBC, bool WIDE, bool SEG, int FR>
__global__ void __launch_bounds__(kFThreads, WIDE ? kFMinBlocks / 2 : kFMinBlocks) ssm_fwd_kernel(const __grid_constant__ FwdLaunch P) {
  using S = FwdSmem<T, TBC>;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  int* bcast = reinterpret_cast<int*>(smem + S::kBars + 16 * kFStages);  // ticket, lookback flag

  // CTA identity: with segments, from an atomic ticket in scan order (first
  // segments first, so every segment a CTA waits for is already running);
  // otherwise from the block index.  Grid: (channel tiles, batch, directions x segments).
  int tile = blockIdx.x, b = blockIdx.y, dz = blockIdx.z;
  if (SEG) {
    if (threadIdx.x == 0) bcast[0] = atomicAdd(P.ticket, 1);
    __syncthreads();
    const int k = bcast[0];
    const int r = k % P.chains;
    tile = r % P.ntile;
    b = (r / P.ntile) % P.batch;
    dz = (r / (P.ntile * P.batch)) * P.zdiv + k / P.chains;
  }
  const FwdDir& a = P.dir[dz / P.zdiv];
  const int seg = dz % P.zdiv;
  const int c0 = tile * kTileCh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = lane & 3;
  const int cl = warp * 8 + (lane >> 2);
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;
  constexpr bool FAST = FR != 0;
  const bool rev = FR == 2 || (FR == 0 && (a.flags & SSM_REVERSE) != 0);
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool aligned = (a.flags & SSM_ALIGNED_SKIP) != 0;
  const bool softplus = FAST || (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  const bool has_z = a.has_z != 0, has_D = a.D != nullptr;
  const bool need_uo = has_D && rev && !aligned;
  const int nblk = (L + kChunk - 1) / kChunk;
  const int nck = (L + kCk - 1) / kCk;
  const int j0 = seg * a.seg_chunks;
  const int j1 = min(nblk, j0 + a.seg_chunks);
  const int nloc = j1 - j0;
  const bool cvalid = FAST || c < Dm;
  const int co = comp ? Dm - 1 - c : c;
  const int oc0 = comp ? Dm - kTileCh - c0 : c0;
  // Loads: first the aggregate pass over the segment (segments that a later
  // CTA waits for; u, delta, B only), then the main pass; load g uses stage
  // g % kFStages.
  constexpr bool lookback = SEG;
  const int nagg = (lookback && seg < a.nseg - 1) ? nloc : 0;
  const int ntot = nagg + nloc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&bars[s], 1);                            // full: the TMA loads of the stage landed
      mbar_init(&bars[kFStages + s], kFThreads / 32);    // empty: every warp is done with the stage
    }
    fence_mbar_init();
  }
  __syncthreads();

  const uint32_t tx_agg = 2 * S::kAct + S::kBC;
  const uint32_t tx = 2 * S::kAct + 2 * S::kBC + (has_z ? S::kAct : 0) + (need_uo ? S::kAct : 0);
  auto issue = [&](int g) {
    const bool ag = g < nagg;
    unsigned char* st = smem + (g % kFStages) * S::kStage;
    uint64_t* bar = &bars[g % kFStages];
    const int t0 = (j0 + (ag ? g : g - nagg)) * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, ag ? tx_agg : tx);
    tma_load_3d(st + S::kOffU, &a.tm_u, bar, c0, t0, b);
    tma_load_3d(st + S::kOffDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S::kOffB, &a.tm_B, bar, 0, t0, b);
    if (!ag) {
      tma_load_3d(st + S::kOffC, &a.tm_C, bar, 0, t0, b);
      if (has_z) tma_load_3d(st + S::kOffZ, &a.tm_z, bar, oc0, ot0, b);
      if (need_uo) tma_load_3d(st + S::kOffUo, &a.tm_u, bar, oc0, ot0, b);
    }
  };
  if (threadIdx.x == 0) {
    const int npre = ntot < kFStages ? ntot : kFStages;
    for (int g = 0; g < npre; ++g) issue(g);
  }

  float2 A2[2];
  {
    const float4 v = cvalid ? *reinterpret_cast<const float4*>(a.A + (size_t)c * kN + 4 * nq)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    A2[0] = make_float2(v.x * kLog2e, v.y * kLog2e);
    A2[1] = make_float2(v.z * kLog2e, v.w * kLog2e);
  }
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsk = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;
  float2 h[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float tsum = 0.f;
  T* out = reinterpret_cast<T*>(a.out);
  const bool b1 = (nq & 2) != 0, b0 = (nq & 1) != 0;
  bool failed = false;

  // One 16-step stage (load g, chunk j).  AGG: the recurrence only (no y,
  // checkpoints or outputs).  Returns false if a bounded wait gave up.
  auto run_stage = [&](auto agg_c, int g) -> bool {
    constexpr bool AGG = decltype(agg_c)::value;
    const int j = j0 + (AGG ? g : g - nagg);
    const int s = g % kFStages;
    const bool ok = mbar_wait_bounded(&bars[s], (g / kFStages) & 1);
    if (!__all_sync(kFull, ok)) return false;  // warps proceed independently
    const unsigned char* st = smem + s * S::kStage;
    const T* su = reinterpret_cast<const T*>(st + S::kOffU);
    const T* sd = reinterpret_cast<const T*>(st + S::kOffDelta);
    const TBC* sB = reinterpret_cast<const TBC*>(st + S::kOffB) + 4 * nq;
    const TBC* sC = reinterpret_cast<const TBC*>(st + S::kOffC) + 4 * nq;

    float dtv[4], dxv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tl = 4 * i + nq;
      const bool valid = FAST || j * kChunk + tl < L;
      const float x = ld_f(su + tl * kTileCh + cl);
      const float dr = ld_f(sd + tl * kTileCh + cl) + bias;
      float dt = softplus ? softplus_f(dr) : dr;
      dt = valid ? dt : 0.f;
      dtv[i] = dt;
      dxv[i] = valid ? dt * x : 0.f;
      if (AGG) tsum += dt;
    }

    float yv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // 4 steps per group, reduce-scattered over the quad
      float yp[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int tl = 4 * i + k;
        const int src = (lane & ~3) | k;
        const float dt = __shfl_sync(kFull, dtv[i], src);
        const float dx = __shfl_sync(kFull, dxv[i], src);
        const float4 Bv = ld4(sB + tl * kN);
        const float2 dt2 = dup2(dt), dx2 = dup2(dx);
        const float2 e0 = fmul2(A2[0], dt2), e1 = fmul2(A2[1], dt2);
        const float2 al0 = make_float2(ex2(e0.x), ex2(e0.y));
        const float2 al1 = make_float2(ex2(e1.x), ex2(e1.y));
        h[0] = ffma2(al0, h[0], fmul2(make_float2(Bv.x, Bv.y), dx2));
        h[1] = ffma2(al1, h[1], fmul2(make_float2(Bv.z, Bv.w), dx2));
        if (!AGG) {
          const float4 Cv = ld4(sC + tl * kN);
          const float2 y2 = ffma2(make_float2(Cv.z, Cv.w), h[1], fmul2(make_float2(Cv.x, Cv.y), h[0]));
          yp[k] = y2.x + y2.y;
          if ((tl & (kCk - 1)) == kCk - 1) {  // checkpoint after every kCk steps
            const int ck = j * (kChunk / kCk) + tl / kCk;
            if (cvalid && ck < nck)
              *reinterpret_cast<float4*>(a.states + (((size_t)b * nck + ck) * Dm + c) * kN + 4 * nq) =
                  make_float4(h[0].x, h[0].y, h[1].x, h[1].y);
          }
        }
      }
      if (!AGG) {
        // lane bit 1: keep steps {0,1} or {2,3}; lane bit 0: keep one of the two
        const float k0 = b1 ? yp[2] : yp[0], k1 = b1 ? yp[3] : yp[1];
        const float s0 = b1 ? yp[0] : yp[2], s1 = b1 ? yp[1] : yp[3];
        const float r0 = k0 + __shfl_xor_sync(kFull, s0, 2);
        const float r1 = k1 + __shfl_xor_sync(kFull, s1, 2);
        const float kk = b0 ? r1 : r0, ss = b0 ? r0 : r1;
        yv[i] = kk + __shfl_xor_sync(kFull, ss, 1);  // total of step 4 i + nq
      }
    }

    if (!AGG) {  // epilogue of this lane's steps (t = 4 i + nq); gate chosen once per stage
      const T* sz = reinterpret_cast<const T*>(st + S::kOffZ);
      const T* suo = reinterpret_cast<const T*>(st + S::kOffUo);
      auto epilogue = [&](auto gate) {
        constexpr int G = decltype(gate)::value;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tl = 4 * i + nq;
          const int t = j * kChunk + tl;
          const int row = rev ? kChunk - 1 - tl : tl;
          const int col = comp ? kTileCh - 1 - cl : cl;
          const int l = rev ? L - 1 - t : t;
          const float xs = need_uo ? ld_f(suo + row * kTileCh + col) : ld_f(su + tl * kTileCh + cl);
          float y = fmaf(Dsk, xs, yv[i]);
          if (G >= 0) y *= act_f(ld_f(sz + row * kTileCh + col), G);
          if (FAST || (t < L && cvalid)) st_act(out + ((size_t)b * L + l) * a.out_stride + co, y);
        }
      };
      switch (has_z ? a.gate_act : -1) {
        case -1: epilogue(std::integral_constant<int, -1>{}); break;
        case SSM_ACT_SILU: epilogue(std::integral_constant<int, SSM_ACT_SILU>{}); break;
        case SSM_ACT_GELU: epilogue(std::integral_constant<int, SSM_ACT_GELU>{}); break;
        case SSM_ACT_RELU: epilogue(std::integral_constant<int, SSM_ACT_RELU>{}); break;
        default: epilogue(std::integral_constant<int, SSM_ACT_NONE>{}); break;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[kFStages + s]);  // this warp no longer reads stage s
    bool rok = true;
    if (threadIdx.x == 0 && g + kFStages < ntot) {  // refill stage s once every warp released it
      rok = mbar_wait_bounded(&bars[kFStages + s], (g / kFStages) & 1);
      if (rok) {
        fence_proxy_async_smem();
        issue(g + kFStages);
      }
    }
    return __shfl_sync(kFull, rok, 0);  // warp-uniform (lane 0 of warp 0 refills)
  };

  // ---- aggregate pass: this segment's end state from a zero start and its
  // sum of dt, folded by the segments after it (the chunk carry of
  // src/selectssm/selectssm.py:87, 91 and 107).
  for (int g = 0; g < nagg && !failed; ++g) failed = !run_stage(std::true_type{}, g);
  if (lookback) {
    // The state entering this segment is the inclusive end state of the one
    // before it; each segment publishes its own as H + exp(A T) * that state as
    // soon as it knows it.  The aggregate passes of all segments run in
    // parallel and only this short step is chained, always in segment order,
    // so the result does not depend on timing.
    failed = __syncthreads_or(failed);
    tsum += __shfl_xor_sync(kFull, tsum, 1);
    tsum += __shfl_xor_sync(kFull, tsum, 2);
    int* my_flag = a.seg_flag + ((size_t)b * P.ntile + tile) * a.nseg + seg;
    float2 carry[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    if (!failed && seg > 0) {
      if (cta_wait_flag(my_flag - 1, P.spin_limit, bcast + 1) == 0) {
        failed = true;
      } else {
        const size_t row = ((size_t)b * a.nseg + seg - 1) * Dm + (cvalid ? c : 0);
        const float4 X = __ldcg(reinterpret_cast<const float4*>(a.segI + row * kN + 4 * nq));
        carry[0] = make_float2(X.x, X.y);
        carry[1] = make_float2(X.z, X.w);
      }
    }
    if (!failed && nagg) {  // publish the inclusive end state: H + exp(A T) carry
      const float2 t2 = dup2(tsum);
      const float2 e0 = fmul2(A2[0], t2), e1 = fmul2(A2[1], t2);
      const float2 i0 = ffma2(make_float2(ex2(e0.x), ex2(e0.y)), carry[0], h[0]);
      const float2 i1 = ffma2(make_float2(ex2(e1.x), ex2(e1.y)), carry[1], h[1]);
      if (cvalid)
        *reinterpret_cast<float4*>(a.segI + (((size_t)b * a.nseg + seg) * Dm + c) * kN + 4 * nq) =
            make_float4(i0.x, i0.y, i1.x, i1.y);
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) st_release_gpu(my_flag, kInclReady);
    }
    h[0] = carry[0];  // the main pass starts from the true state entering the segment
    h[1] = carry[1];
  }
  // ---- main pass
  for (int g = nagg; g < ntot && !failed; ++g) failed = !run_stage(std::false_type{}, g);
  if (failed && lane == 0) report(a.status, kStatusTimeout);
}

}  // namespace ssm
