// Selective-scan forward kernel for large grids: one lane per channel.
//
// The quad-per-channel forward (scan_fwd.cuh) spreads a channel's 16 states
// over 4 lanes so that a batch of 8 rows still fills the GPU; that costs two
// shuffles per step for the per-step scalars and a reduce-scatter of y over
// the quad.  With many (batch row, channel) pairs, e.g. 64 rows of 1536
// channels, a lane can own a whole channel: the per-step scalars (softplus,
// dt x, the D skip and the gate) are computed once per channel and step with
// no exchange, y = C . h is a sum inside the lane, and the 16 independent
// state updates per step give each warp enough independent work that a few
// warps per scheduler keep the special-function unit (the exponentials) busy.
//
// Work decomposition
//   CTA  = one batch row b x 128 consecutive channels (4 warps); lane = channel.
//   time = TMA stages of 16 steps (u, delta, z tiles of 128 ch x 16 steps; B and
//          C rows of 16 x 16 float32, widened from bf16 beforehand when needed)
//          in a ring of two shared-memory stages completed on mbarriers;
//          thread 0 refills a stage once all four warps released it.
//   B and C rows are read as broadcast float4 loads (every lane of a warp
//   reads the same row).
//
// Serves single-direction, forward-frame launches with softplus(dt), whole
// 16-step chunks and whole 128-channel tiles, without sequence segments: the
// frame, the softplus and the bounds masks are compile-time constants.  The
// gate activation G (an ssm_act code; -1 without z) is a template parameter.
// Recurrence (src/selectssm/selectssm.py:74-78, :90): h_t = exp(A dt_t) h_{t-1}
// + dt_t B_t x_t, y_t = C_t . h_t; then the D skip (:238) and the gate
// y * act(z) (:335-338).  The state after every 8 steps goes to `states`, in
// the same layout the backward reads.
#pragma once

#include "scan_kernels.cuh"

namespace ssm {

#ifndef SSM_LANE_TILE
#define SSM_LANE_TILE 128
#endif
constexpr int kLTile = SSM_LANE_TILE;  // channels per CTA (one per thread)
constexpr int kLThreads = kLTile;
// Channels (batch rows x channels) from which the one-lane kernel is used:
// below this the quad-per-channel kernel fills the GPU better.
#ifndef SSM_LANE_MIN_CHANNELS
#define SSM_LANE_MIN_CHANNELS 65536
#endif
constexpr long kLaneMinChannels = SSM_LANE_MIN_CHANNELS;

template <typename T>
struct LaneSmem {
  static constexpr int kStages = 2;
  static constexpr int kAct = kChunk * kLTile * (int)sizeof(T);
  static constexpr int kBC = kChunk * kN * 4;
  static constexpr int kOffU = 0, kOffDelta = kAct, kOffZ = 2 * kAct, kOffB = 3 * kAct, kOffC = 3 * kAct + kBC;
  static constexpr int kStage = 3 * kAct + 2 * kBC;
  static constexpr int kBars = kStage * kStages;  // full[kStages] then empty[kStages]
  static constexpr int kBytes = kBars + 16 * kStages;
};

// Resident threads per SM the register budget targets: 24 warps (80 registers)
// with bf16 activations, 16 warps (128 registers) with float32 ones.
template <typename T>
constexpr int lane_min_blocks() {
  return (sizeof(T) == 2 ? 768 : 512) / kLThreads;
}

template <typename T, int G>
__global__ void __launch_bounds__(kLThreads, lane_min_blocks<T>())
    ssm_fwd_lane_kernel(const __grid_constant__ FwdLaunch P) {
  using S = LaneSmem<T>;
  constexpr int kStages = S::kStages;
  constexpr bool has_z = G >= 0;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  const FwdDir& a = P.dir[0];
  const int c0 = blockIdx.x * kLTile, b = blockIdx.y;
  const int c = c0 + threadIdx.x;
  const int lane = threadIdx.x & 31;
  constexpr int kWarps = kLThreads / 32;
  const int L = a.L, Dm = a.Dm;
  const int nblk = L / kChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[s], 1);                         // full: the stage's TMA loads landed
      mbar_init(&bars[kStages + s], kWarps);  // empty: every warp is done with it
    }
    fence_mbar_init();
  }
  __syncthreads();

  const uint32_t tx = 2 * S::kAct + 2 * S::kBC + (has_z ? S::kAct : 0);
  auto issue = [&](int g) {
    unsigned char* st = smem + (g % kStages) * S::kStage;
    uint64_t* bar = &bars[g % kStages];
    const int t0 = g * kChunk;
    mbar_arrive_expect_tx(bar, tx);
    tma_load_3d(st + S::kOffU, &a.tm_u, bar, c0, t0, b);
    tma_load_3d(st + S::kOffDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S::kOffB, &a.tm_B, bar, 0, t0, b);
    tma_load_3d(st + S::kOffC, &a.tm_C, bar, 0, t0, b);
    if (has_z) tma_load_3d(st + S::kOffZ, &a.tm_z, bar, c0, t0, b);
  };
  if (threadIdx.x == 0) {
    const int npre = nblk < kStages ? nblk : kStages;
    for (int g = 0; g < npre; ++g) issue(g);
  }

  float2 A2[8];  // A log2(e)
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = *reinterpret_cast<const float4*>(a.A + (size_t)c * kN + 4 * q);
    A2[2 * q] = make_float2(v.x * kLog2e, v.y * kLog2e);
    A2[2 * q + 1] = make_float2(v.z * kLog2e, v.w * kLog2e);
  }
  const float bias = a.bias ? a.bias[c] : 0.f;
  const float Dsk = a.D ? a.D[c] : 0.f;
  float2 h[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) h[p] = make_float2(0.f, 0.f);
  T* out = reinterpret_cast<T*>(a.out) + (size_t)b * L * a.out_stride + c;
  float* ckp = a.states + ((size_t)b * (L / kCk) * Dm + c) * kN;
  bool failed = false;

  for (int g = 0; g < nblk; ++g) {
    const int s = g % kStages;
    const bool ok = mbar_wait_bounded(&bars[s], (g / kStages) & 1);
    if (!__all_sync(kFull, ok)) {
      failed = true;
      break;
    }
    const unsigned char* st = smem + s * S::kStage;
    const T* su = reinterpret_cast<const T*>(st + S::kOffU) + threadIdx.x;
    const T* sd = reinterpret_cast<const T*>(st + S::kOffDelta) + threadIdx.x;
    const T* sz = reinterpret_cast<const T*>(st + S::kOffZ) + threadIdx.x;
    const float* sB = reinterpret_cast<const float*>(st + S::kOffB);
    const float* sC = reinterpret_cast<const float*>(st + S::kOffC);
#pragma unroll
    for (int tl = 0; tl < kChunk; ++tl) {
      const float x = ld_f(su + tl * kLTile);
      const float dt = softplus_f(ld_f(sd + tl * kLTile) + bias);
      const float2 dt2 = dup2(dt), dx2 = dup2(dt * x);
      float2 y2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // two chains
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 Bv = *reinterpret_cast<const float4*>(sB + tl * kN + 4 * q);
        const float4 Cv = *reinterpret_cast<const float4*>(sC + tl * kN + 4 * q);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int p = 2 * q + k;
          const float2 e = fmul2(A2[p], dt2);
          const float2 al = make_float2(ex2(e.x), ex2(e.y));
          const float2 Bp = k ? make_float2(Bv.z, Bv.w) : make_float2(Bv.x, Bv.y);
          const float2 Cp = k ? make_float2(Cv.z, Cv.w) : make_float2(Cv.x, Cv.y);
          h[p] = ffma2(al, h[p], fmul2(Bp, dx2));
          y2[q >> 1] = ffma2(Cp, h[p], y2[q >> 1]);
        }
      }
      const float2 ys = fadd2(y2[0], y2[1]);
      float y = fmaf(Dsk, x, ys.x + ys.y);
      if (has_z) y *= act_f(ld_f(sz + tl * kLTile), G);
      st_act(out + (size_t)(g * kChunk + tl) * a.out_stride, y);
      if ((tl & (kCk - 1)) == kCk - 1) {  // checkpoint after every kCk steps
        float4* dst = reinterpret_cast<float4*>(ckp + (size_t)(g * (kChunk / kCk) + tl / kCk) * Dm * kN);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_float4(h[2 * q].x, h[2 * q].y, h[2 * q + 1].x, h[2 * q + 1].y);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[kStages + s]);  // this warp no longer reads stage s
    bool rok = true;
    if (threadIdx.x == 0 && g + kStages < nblk) {  // refill stage s once every warp released it
      rok = mbar_wait_bounded(&bars[kStages + s], (g / kStages) & 1);
      if (rok) {
        fence_proxy_async_smem();
        issue(g + kStages);
      }
    }
    if (!__shfl_sync(kFull, rok, 0)) {  // warp-uniform (thread 0 refills)
      failed = true;
      break;
    }
  }
  if (failed && lane == 0) report(a.status, kStatusTimeout);
}

}  // namespace ssm
