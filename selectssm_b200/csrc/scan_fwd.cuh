// Selective-scan forward kernel for B200 (sm_100a), lane-pair design.
//
// Work decomposition
//   CTA   = one batch row b x 32 consecutive channels x one sequence segment;
//           2 warps of 16 channels.  A channel belongs to a lane pair
//           (lane = 2 ch + half); each lane owns 8 of the 16 states
//           (n = 8 half .. 8 half + 7) as 4 packed f32x2 pairs.
//   time  = TMA stages of 16 steps (u, delta, z tiles of 32 ch x 16 steps, the
//           B and C tiles of 16 steps x 16 states) in a ring of shared-memory
//           stages completed on mbarriers, issued STAGES-1 stages ahead.
//   Per stage, each lane evaluates the per-step scalars softplus(dt + bias) and
//   dt x for the 8 steps of its parity (t = 2 i + half) and the pair swaps them
//   with one shuffle each per step.  y_t = C_t . h_t is half on each lane; one
//   shuffle per two steps both completes it and hands step 2i to half 0 and
//   step 2i+1 to half 1, which run the epilogue (D skip, gate, store) for the
//   steps they own.
//   alpha = 2^(A log2(e) dt) uses the MUFU unit for 4 - EMU pairs and the FMA
//   pipe (ex2_poly2) for EMU pairs, so the two units share the exponentials.
//
// Recurrence (src/selectssm/selectssm.py:74-78, :90): h_t = exp(A dt_t) h_{t-1}
// + dt_t B_t x_t, y_t = C_t . h_t; then the D skip (:238), the reverse /
// complement unflip (:230-231) and the gate y * act(z) (:335-338).  The state
// after every 8 steps is written to `states` for the backward.
//
// AGG: the segment pre-pass.  It runs one segment from a zero state and writes
// only the segment's end state and its sum of dt; the main pass starts segment
// s from the end states of segments 0..s-1 folded together
// (h <- exp(A sum dt) h + H).
#pragma once

#include <type_traits>

#include "scan_kernels.cuh"

namespace ssm {

constexpr int kFThreads = 64;      // 2 warps x 16 channels = kTileCh
constexpr int kFStages = 3;
constexpr int kFEmu = 1;           // state pairs per lane whose exponential runs on the FMA pipe

template <typename T, typename TBC>
struct FwdSmem2 {
  static constexpr int kAct = kChunk * kTileCh * (int)sizeof(T);
  static constexpr int kBC = kChunk * kN * (int)sizeof(TBC);
  static constexpr int kOffU = 0, kOffDelta = kAct, kOffZ = 2 * kAct, kOffUo = 3 * kAct;
  static constexpr int kOffB = 4 * kAct, kOffC = 4 * kAct + kBC;
  static constexpr int kStage = 4 * kAct + 2 * kBC;
  static constexpr int kBars = kStage * kFStages;
  static constexpr int kBytes = kBars + 8 * kFStages;
};

template <typename TB>
__device__ __forceinline__ void ld8(const TB* row, float2 (&v)[4]) {
  const float4 a = ld4(row), b = ld4(row + 4);
  v[0] = make_float2(a.x, a.y);
  v[1] = make_float2(a.z, a.w);
  v[2] = make_float2(b.x, b.y);
  v[3] = make_float2(b.z, b.w);
}

template <typename T, typename TBC, bool AGG, int EMU>
__global__ void __launch_bounds__(kFThreads, 8) ssm_fwd2_kernel(const __grid_constant__ FwdLaunch P) {
  using S = FwdSmem2<T, TBC>;
  const FwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = blockIdx.z % P.zdiv;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kTileCh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane & 1;
  const int cl = warp * 16 + (lane >> 1);
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
  const int co = comp ? Dm - 1 - c : c;              // output-frame channel
  const int oc0 = comp ? Dm - kTileCh - c0 : c0;     // output-frame tile start

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const uint32_t tx = AGG ? 2 * S::kAct + S::kBC
                          : 2 * S::kAct + 2 * S::kBC + (has_z ? S::kAct : 0) + (need_uo ? S::kAct : 0);
  auto issue = [&](int jl) {  // local stage index within the segment
    unsigned char* st = smem + (jl % kFStages) * S::kStage;
    uint64_t* bar = &bars[jl % kFStages];
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
    const int npre = nloc < kFStages ? nloc : kFStages;
    for (int jl = 0; jl < npre; ++jl) issue(jl);
  }

  // per-lane constants: A log2(e) of this lane's 8 states
  float2 A2[4];
  {
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    if (cvalid) {
      a0 = *reinterpret_cast<const float4*>(a.A + (size_t)c * kN + half * 8);
      a1 = *reinterpret_cast<const float4*>(a.A + (size_t)c * kN + half * 8 + 4);
    }
    A2[0] = make_float2(a0.x * kLog2e, a0.y * kLog2e);
    A2[1] = make_float2(a0.z * kLog2e, a0.w * kLog2e);
    A2[2] = make_float2(a1.x * kLog2e, a1.y * kLog2e);
    A2[3] = make_float2(a1.z * kLog2e, a1.w * kLog2e);
  }
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsk = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;
  float2 h[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) h[p] = make_float2(0.f, 0.f);
  if (!AGG && cvalid) {  // fold the end states of the preceding segments
    for (int sp = 0; sp < seg; ++sp) {
      const size_t r = (size_t)b * a.nseg + sp;
      const float Tsum = a.segT[r * Dm + c];
      float2 H[4];
      ld8(a.segH + (r * Dm + c) * kN + half * 8, H);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 e = fmul2(A2[p], dup2(Tsum));
        h[p] = ffma2(make_float2(ex2(e.x), ex2(e.y)), h[p], H[p]);
      }
    }
  }
  float tsum = 0.f;  // AGG: sum of dt over this lane's steps
  T* out = reinterpret_cast<T*>(a.out);

  for (int j = j0; j < j1; ++j) {
    const int jl = j - j0;
    const int s = jl % kFStages;
    const bool ok = mbar_wait_bounded(&bars[s], (jl / kFStages) & 1);
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) report(a.status, kStatusTimeout);
      return;
    }
    const unsigned char* st = smem + s * S::kStage;
    const T* su = reinterpret_cast<const T*>(st + S::kOffU);
    const T* sd = reinterpret_cast<const T*>(st + S::kOffDelta);
    const TBC* sB = reinterpret_cast<const TBC*>(st + S::kOffB);
    const TBC* sC = reinterpret_cast<const TBC*>(st + S::kOffC);

    // per-step scalars of this lane's 8 steps (tl = 2 i + half)
    float dtv[8], dxv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int tl = 2 * i + half;
      const bool valid = j * kChunk + tl < L;
      const float x = ld_f(su + tl * kTileCh + cl);
      const float dr = ld_f(sd + tl * kTileCh + cl) + bias;
      float dt = softplus ? softplus_f(dr) : dr;
      dt = valid ? dt : 0.f;
      dtv[i] = dt;
      dxv[i] = valid ? dt * x : 0.f;
      tsum += dt;
    }

    float yv[8];
    float yeven = 0.f;
#pragma unroll
    for (int tl = 0; tl < kChunk; ++tl) {
      const int src = (lane & ~1) | (tl & 1);
      const float dt = __shfl_sync(kFull, dtv[tl >> 1], src);
      const float dx = __shfl_sync(kFull, dxv[tl >> 1], src);
      float2 Bq[4];
      ld8(sB + tl * kN + half * 8, Bq);
      const float2 dt2 = dup2(dt), dx2 = dup2(dx);
      float2 alpha[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 e = fmul2(A2[p], dt2);
        alpha[p] = p < EMU ? ex2_poly2(e) : make_float2(ex2(e.x), ex2(e.y));
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) h[p] = ffma2(alpha[p], h[p], fmul2(Bq[p], dx2));
      if (!AGG) {
        float2 Cq[4];
        ld8(sC + tl * kN + half * 8, Cq);
        float2 y2 = fmul2(Cq[0], h[0]);
#pragma unroll
        for (int p = 1; p < 4; ++p) y2 = ffma2(Cq[p], h[p], y2);
        const float yp = y2.x + y2.y;
        if ((tl & 1) == 0) {
          yeven = yp;
        } else {  // half 0 keeps step tl-1, half 1 keeps step tl
          const float mine = half ? yp : yeven, other = half ? yeven : yp;
          yv[tl >> 1] = mine + __shfl_xor_sync(kFull, other, 1);
        }
        if ((tl & (kCk - 1)) == kCk - 1) {  // checkpoint after every kCk steps
          const int ck = j * (kChunk / kCk) + tl / kCk;
          if (cvalid && ck < nck) {
            float4* sp = reinterpret_cast<float4*>(a.states + (((size_t)b * nck + ck) * Dm + c) * kN + half * 8);
            sp[0] = make_float4(h[0].x, h[0].y, h[1].x, h[1].y);
            sp[1] = make_float4(h[2].x, h[2].y, h[3].x, h[3].y);
          }
        }
      }
    }

    if (!AGG) {  // epilogue: skip, gate, store (this lane's 8 steps); gate chosen once per stage
      const T* sz = reinterpret_cast<const T*>(st + S::kOffZ);
      const T* suo = reinterpret_cast<const T*>(st + S::kOffUo);
      auto epilogue = [&](auto gate) {
        constexpr int G = decltype(gate)::value;  // -1: no z, else an ssm_act code
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tl = 2 * i + half;
          const int t = j * kChunk + tl;
          const int row = rev ? kChunk - 1 - tl : tl;
          const int col = comp ? kTileCh - 1 - cl : cl;
          const int l = rev ? L - 1 - t : t;
          const float xs = need_uo ? ld_f(suo + row * kTileCh + col) : ld_f(su + tl * kTileCh + cl);
          float y = fmaf(Dsk, xs, yv[i]);
          if (G >= 0) y *= act_f(ld_f(sz + row * kTileCh + col), G);
          if (t < L && cvalid) st_act(out + ((size_t)b * L + l) * a.out_stride + co, y);
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
    __syncthreads();  // both warps are done with stage s
    if (threadIdx.x == 0 && jl + kFStages < nloc) {
      fence_proxy_async_smem();
      issue(jl + kFStages);
    }
  }
  if (AGG) {
    tsum += __shfl_xor_sync(kFull, tsum, 1);
    if (cvalid) {
      const size_t r = (size_t)b * a.nseg + seg;
      float4* hp = reinterpret_cast<float4*>(a.segH + (r * Dm + c) * kN + half * 8);
      hp[0] = make_float4(h[0].x, h[0].y, h[1].x, h[1].y);
      hp[1] = make_float4(h[2].x, h[2].y, h[3].x, h[3].y);
      if (half == 0) a.segT[r * Dm + c] = tsum;
    }
  }
}

}  // namespace ssm
