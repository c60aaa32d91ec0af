// Selective-scan backward kernel for B200 (sm_100a).
//
// Work decomposition
//   CTA   = one batch row b x 128 consecutive channels x one sequence segment;
//           8 warps of 16 channels.  A channel belongs to two lanes of its
//           warp (lane = 16 hs + channel), each owning 8 of the 16 states
//           (hs = 0: states 0-7, hs = 1: states 8-15) as 4 packed f32x2 pairs,
//           so a thread holds half the state of a lane-per-channel layout and
//           twice as many warps fit on an SM (16, at most 128 registers).
//   time  = TMA stages of 16 steps (u, delta, dout, z tiles of 128 ch x 16
//           steps; B and C tiles of 16 x 16), double buffered on mbarriers and
//           visited last to first; each stage is two 8-step blocks, last first.
//   block = per-step scalars first: the two lanes of a channel each evaluate
//           softplus(dt), dt*x and the gated upstream gradient for one step of
//           every step pair and swap them (one shuffle each), so the scalar work
//           is not duplicated.  Then restart from the state the forward saved
//           before the block (plain 128-bit loads), recompute alpha_t = exp(A dt_t)
//           and alpha_t h_{t-1} for the 8 steps into tensor memory (TMEM: 8 steps
//           x 16 values = 128 columns per lane; warps 0-3 and 4-7 share the 128
//           TMEM lanes and use column halves), then run the adjoint
//           f_t = alpha_{t+1} f_{t+1} + C_t dy_t backwards reading them back.
//           Sums over states (y, sum_n f B, sum_n f A alpha h) add the two
//           halves with one shuffle; each lane then finishes the per-step
//           epilogue (du, ddelta, dz stores) of its own step of every pair.
//   Leaf gradients (src/selectssm/ssmrecscan.py:150-161):
//     dx_t = dt_t sum_n f B_t,  dA += dt_t f alpha_t h_{t-1},  dB_t = sum_d dt_t x_t f,
//     dC_t = sum_d dy_t h_t,    ddt_t = sum_n f (A alpha_t h_{t-1} + B_t x_t).
//   dB / dC (sums over channels) use a shuffle reduce-scatter over the 16
//   channels of a half-warp.  Lanes hold their two state quads in an order
//   swapped by lane bit 3, so the first exchange needs no selects.  The 8
//   warps' partials are summed in shared memory and stored as this channel
//   tile's partial; the finalize kernel sums the tiles in a fixed order, so
//   dB / dC are bit-reproducible.  dA/dD/d(delta_bias) are per-(batch row,
//   segment) partials summed in a fixed order by the finalize kernel.
//   The gate activation is a template parameter (fixed per launch) and the
//   per-step work holds no data- or flag-dependent branch (only stores are
//   predicated), so the compiler can schedule across the unrolled steps.
// Segments: with few (batch row, channel tile) chains the sequence is cut into
//   segments run by separate CTAs of one launch.  A CTA takes its segment from
//   an atomic ticket, last segment first.  A segment that an earlier one
//   depends on first runs the adjoint over its own steps from a zero carry
//   (the aggregate pass: delta, C, dout, z only), keeping that carry and its
//   sum of dt in registers; it then waits (bounded) for the inclusive carry of
//   the segment after it, publishes its own (F + exp(A T) carry) under a flag
//   and runs the main pass from the true carry.  Only that short step is
//   chained, in segment order, so the result does not depend on timing.
#pragma once

#include "scan_kernels.cuh"

namespace ssm {

constexpr int kBTile = 128;                            // channels per backward CTA
constexpr int kBWarps = kBTile / 16;                   // 16 channels per warp
constexpr int kBThreads = 2 * kBTile;
constexpr int kBStages = 2;
constexpr uint32_t kBTmemCols = 2 * kCk * kN;          // 2 warp groups x 8 steps x (8 alpha + 8 alpha*h)

// Shared-memory layout (bytes), sized at run time: the output-frame copy of u
// and the scan-frame copies of dout / z only exist for the reverse direction
// with the reference's skip frame.
struct BwdLayout {
  int offU, offDelta, offDo, offZo, offUo, offDs, offZs, offB, offC, stage;
  int offRed, offBars, offTmem, bytes;
  __host__ __device__ BwdLayout(int es, int esbc, bool has_z, bool mirror) {
    const int act = kChunk * kBTile * es, bc = kChunk * kN * esbc;
    int o = 0;
    offU = o; o += act;
    offDelta = o; o += act;
    offDo = o; o += act;
    offZo = o; if (has_z) o += act;
    offUo = o; if (mirror) o += act;
    offDs = o; if (mirror) o += act;
    offZs = o; if (mirror && has_z) o += act;
    offB = o; o += bc;
    offC = o; o += bc;
    stage = (o + 127) & ~127;
    offRed = stage * kBStages;                              // two [warp][step][32] partial buffers
    offBars = offRed + 2 * kBWarps * kChunk * 32 * 4;
    offTmem = offBars + 8 * kBStages;
    bytes = offTmem + 16;
  }
  // The CTA's ticket is broadcast through the first word of shared memory
  // (stage 0's u tile): it is read before the first TMA load is issued.
  static constexpr int kTicketSlot = 0;
  __host__ __device__ static uint32_t tx(int es, int esbc, bool has_z, bool mirror) {
    const int act = kChunk * kBTile * es, bc = kChunk * kN * esbc;
    return 3 * act + 2 * bc + (has_z ? act : 0) + (mirror ? (has_z ? 3 : 2) * act : 0);
  }
};

// Sum over the 16 channel-lanes of a half-warp of a lane's 8 per-state values
// (4 packed pairs).  Pair slot p holds states 8 hs + 4 ((p >> 1) ^ b3) +
// 2 (p & 1) + {0, 1} (b3 = lane bit 3).  The result is the total for state
// 8 hs + 4 b3 + 2 b2 + b1 (lane bits 2 and 1); lanes differing in bit 0 hold
// the same total.
__device__ __forceinline__ float reduce16ch(const float2 (&v)[4], bool b2, bool b1) {
  float2 r[2];
#pragma unroll
  for (int p = 0; p < 2; ++p)  // lane bit 3: keep quad slot 0, receive the partner's quad slot 1
    r[p] = fadd2(v[p], make_float2(__shfl_xor_sync(kFull, v[p + 2].x, 8), __shfl_xor_sync(kFull, v[p + 2].y, 8)));
  // lane bit 2: keep one pair of the quad
  const float2 kp = b2 ? r[1] : r[0], sd = b2 ? r[0] : r[1];
  const float2 s = fadd2(kp, make_float2(__shfl_xor_sync(kFull, sd.x, 4), __shfl_xor_sync(kFull, sd.y, 4)));
  // lane bit 1: keep one element of the pair
  float q = (b1 ? s.y : s.x) + __shfl_xor_sync(kFull, b1 ? s.x : s.y, 2);
  q += __shfl_xor_sync(kFull, q, 1);  // lane bit 0: both lanes keep the total
  return q;
}

// This lane's 8 per-state values (states 8 hs .. 8 hs + 7, quads swapped by
// lane bit 3) -> 4 pairs.  `row` points at state 0 of a 16-state row; `q0` is
// the offset of quad slot 0 (8 hs + 4 b3), slot 1 is at q0 ^ 4.
template <typename TB>
__device__ __forceinline__ void ld8q(const TB* row, int q0, float2 (&v)[4]) {
  const float4 f0 = ld4(row + q0), f1 = ld4(row + (q0 ^ 4));
  v[0] = make_float2(f0.x, f0.y);
  v[1] = make_float2(f0.z, f0.w);
  v[2] = make_float2(f1.x, f1.y);
  v[3] = make_float2(f1.z, f1.w);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// TMEM store / load without a memory clobber, so the compiler may move
// shared-memory loads and shuffles across them; a load's registers are tied
// to the wait that completes it (tmem_wait_ld_regs), so no use of them can be
// scheduled before that wait.
__device__ __forceinline__ void tmem_st16_nc(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])));
}
__device__ __forceinline__ void tmem_ld16_nc(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void sts_nc(float* p, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(smem_u32(p)), "f"(v));
}
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}

// G: the gate activation (an ssm_act code; -1 without z), fixed per launch so
// the step loops hold no branch on it.
// MC: dB / dC partial sums go to NVLink multicast addresses (cross-GPU sum);
// a template parameter so the single-GPU instance carries no trace of it.
// SEG: segment code (ticket, aggregate pass, carry chain) compiled in.
template <typename T, typename TBC, int G, bool MC, int FR, bool SEG>
__global__ void __launch_bounds__(kBThreads, 2) ssm_bwd_kernel(const __grid_constant__ BwdLaunch P) {
  extern __shared__ __align__(1024) unsigned char smem[];
  // CTA identity: with segments, from an atomic ticket in scan order (the last
  // segments first, so every segment a CTA waits for is already running);
  // otherwise from the block index.  Grid: (channel tiles, batch, directions x segments).
  int tile = blockIdx.x, b = blockIdx.y, dz = blockIdx.z;
  if (SEG && P.ticket) {
    int* slot = reinterpret_cast<int*>(smem + BwdLayout::kTicketSlot);
    if (threadIdx.x == 0) *slot = atomicAdd(P.ticket, 1) + P.ticket_base;
    __syncthreads();
    const int k = *slot;
    const int r = k % P.chains;
    tile = r % P.ntile;
    b = (r / P.ntile) % P.batch;
    dz = (r / (P.ntile * P.batch)) * P.zdiv + (P.zdiv - 1 - k / P.chains);
  }
  const BwdDir& a = P.dir[dz / P.zdiv];
  const int seg = dz % P.zdiv;

  const int c0 = tile * kBTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hs = lane >> 4;                   // state half of this lane
  const int cl = warp * 16 + (lane & 15);     // channel within the tile
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;
  // FR: 1 (2) = a single-direction forward-frame (reverse-frame) launch with
  // softplus(dt), whose length is a whole number of 16-step chunks and whose
  // channels fill whole 128-channel tiles: frame, softplus and masks are
  // compile-time constants, so the per-step code carries no frame-dependent
  // address selects and no bounds predicates; 0 = generic.  G < 0: no gate.
  constexpr bool FAST = FR != 0;
  const bool rev = FR == 2 || (FR == 0 && (a.flags & SSM_REVERSE) != 0);
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool aligned = (a.flags & SSM_ALIGNED_SKIP) != 0;
  const bool softplus = FAST || (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  constexpr bool has_z = G >= 0;
  const bool has_D = a.D != nullptr;
  const bool mirror = has_D && rev && !aligned;  // skip frame of the reverse direction
  const int nblk = (L + kChunk - 1) / kChunk;
  const int nck = (L + kCk - 1) / kCk;
  const int j1 = min(nblk, (seg + 1) * a.seg_chunks);
  const int nloc = j1 - seg * a.seg_chunks;
  const bool cvalid = FAST || c < Dm;
  const int co = comp ? Dm - 1 - c : c;
  const int oc0 = comp ? Dm - kBTile - c0 : c0;
  const int col = comp ? kBTile - 1 - cl : cl;
  const BwdLayout S(sizeof(T), sizeof(TBC), has_z, mirror);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.offBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S.offTmem);
  float* sRed = reinterpret_cast<float*>(smem + S.offRed);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kBTmemCols);
  tmem_fence_before_sync();
  __syncthreads();
  tmem_fence_after_sync();
  const uint32_t tbase = *tmem_slot;
  // this warp's lane quarter and column half
  const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * kCk * kN);

  // Loads: first the aggregate pass over the segment (segments that a later
  // CTA waits for; delta, C, dout, z only), then the main pass, each visiting
  // the chunks last to first; load g uses stage g % 2.
  const bool lookback = SEG && a.nseg > 1;
  const int nagg = (lookback && seg > 0) ? nloc : 0;
  const int ntot = nagg + nloc;
  const uint32_t tx = BwdLayout::tx(sizeof(T), sizeof(TBC), has_z, mirror);
  const uint32_t tx_agg = 2 * kChunk * kBTile * (int)sizeof(T) + kChunk * kN * (int)sizeof(TBC) +
                          (has_z ? kChunk * kBTile * (int)sizeof(T) : 0);
  auto issue = [&](int g) {
    const bool ag = g < nagg;
    const int j = j1 - 1 - (ag ? g : g - nagg);
    unsigned char* st = smem + (g % kBStages) * S.stage;
    uint64_t* bar = &bars[g % kBStages];
    const int t0 = j * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, ag ? tx_agg : tx);
    tma_load_3d(st + S.offDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S.offC, &a.tm_C, bar, 0, t0, b);
    tma_load_3d(st + S.offDo, &a.tm_dout, bar, oc0, ot0, b);
    if (has_z) tma_load_3d(st + S.offZo, &a.tm_z, bar, oc0, ot0, b);
    if (ag) return;
    tma_load_3d(st + S.offU, &a.tm_u, bar, c0, t0, b);
    tma_load_3d(st + S.offB, &a.tm_B, bar, 0, t0, b);
    if (mirror) {
      tma_load_3d(st + S.offUo, &a.tm_u, bar, oc0, ot0, b);
      tma_load_3d(st + S.offDs, &a.tm_dout, bar, c0, t0, b);
      if (has_z) tma_load_3d(st + S.offZs, &a.tm_z, bar, c0, t0, b);
    }
  };
  if (threadIdx.x == 0) {
    const int npre = ntot < kBStages ? ntot : kBStages;
    for (int g = 0; g < npre; ++g) issue(g);
  }

  // state layout (see reduce16ch / ld8q)
  const bool b3 = ((lane >> 3) & 1) != 0, b2 = ((lane >> 2) & 1) != 0, b1 = ((lane >> 1) & 1) != 0;
  const int q0 = 8 * hs + (b3 ? 4 : 0);
  const int red_n = q0 + (b2 ? 2 : 0) + (b1 ? 1 : 0);
  const bool red_writer = (lane & 1) == 0;
  const bool own_odd = hs != 0;  // this lane finishes the odd step of every step pair
  float2 A2[4];  // A log2(e), this lane's states
  {
    float2 Av[4];
    const float* Arow = a.A + (size_t)(cvalid ? c : 0) * kN;
    ld8q(Arow, q0, Av);
#pragma unroll
    for (int p = 0; p < 4; ++p) A2[p] = fmul2(Av[p], dup2(kLog2e));
  }
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsc = (has_D && cvalid) ? a.D[c] : 0.f;                  // skip weight, scan channel
  const float Dso = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;   // skip weight in the pre-gate value
  float2 fa[4], dA[4];  // f_{t+1} alpha_{t+1} carried backwards; dA accumulators (A log2 e frame)
#pragma unroll
  for (int p = 0; p < 4; ++p) fa[p] = dA[p] = make_float2(0.f, 0.f);
  float dD_acc = 0.f, db_acc = 0.f;
  T* du_g = reinterpret_cast<T*>(a.du) + (size_t)b * L * Dm + c;
  T* dd_g = reinterpret_cast<T*>(a.ddelta) + (size_t)b * L * Dm + c;
  T* dz_g = reinterpret_cast<T*>(a.dz) + (size_t)b * L * a.z_stride + co;
  const float* st_b = a.states + ((size_t)b * nck * Dm + (cvalid ? c : 0)) * kN;
  bool failed = false;

  // ---- aggregate pass: the adjoint over this segment from a zero carry; the
  // carry it leaves at the segment's first step and the segment's sum of dt
  // are what the segment before it folds in (src/selectssm/ssmrecscan.py:121-133
  // chains chunk adjoints the same way).
  float tsum = 0.f;
  for (int g = 0; g < nagg; ++g) {
    const int j = j1 - 1 - g;
    const int s = g % kBStages;
    const bool ok = mbar_wait_bounded(&bars[s], (g / kBStages) & 1);
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    const unsigned char* st = smem + s * S.stage;
    const T* sd = reinterpret_cast<const T*>(st + S.offDelta) + cl;
    const T* szo = reinterpret_cast<const T*>(st + S.offZo) + col;
    const T* sdo = reinterpret_cast<const T*>(st + S.offDo) + col;
    const TBC* sC = reinterpret_cast<const TBC*>(st + S.offC);
#pragma unroll 1
    for (int blk = 1; blk >= 0; --blk) {
      const int T0 = blk * kCk;
      float dtv[kCk], dyv[kCk];
#pragma unroll
      for (int k = 0; k < kCk / 2; ++k) {
        const int tl = T0 + 2 * k + hs;
        const bool valid = FAST || j * kChunk + tl < L;
        const float dr = ld_f(sd + tl * kBTile) + bias;
        float dt = softplus ? softplus_f(dr) : dr;
        dt = valid ? dt : 0.f;
        tsum += dt;
        const int row = rev ? kChunk - 1 - tl : tl;
        float gv = ld_f(sdo + row * kBTile);
        if (has_z) gv *= act_f(ld_f(szo + row * kBTile), G);
        const float dy = valid ? gv : 0.f;
        const float pdt = __shfl_xor_sync(kFull, dt, 16);
        const float pdy = __shfl_xor_sync(kFull, dy, 16);
        dtv[2 * k] = own_odd ? pdt : dt;
        dtv[2 * k + 1] = own_odd ? dt : pdt;
        dyv[2 * k] = own_odd ? pdy : dy;
        dyv[2 * k + 1] = own_odd ? dy : pdy;
      }
#pragma unroll
      for (int u = kCk - 1; u >= 0; --u) {
        float2 Cq[4];
        ld8q(sC + (T0 + u) * kN, q0, Cq);
        const float2 dt2 = dup2(dtv[u]), dy2 = dup2(dyv[u]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 e = fmul2(A2[p], dt2);
          fa[p] = fmul2(ffma2(Cq[p], dy2, fa[p]), make_float2(ex2(e.x), ex2(e.y)));
        }
      }
    }
    __syncthreads();  // stage s consumed
    if (threadIdx.x == 0 && g + kBStages < ntot) {
      fence_proxy_async_smem();
      issue(g + kBStages);
    }
  }
  int* wait_slot = reinterpret_cast<int*>(smem + S.offTmem + 8);
  if (lookback) {
    // The adjoint entering this segment (at its last step) is the inclusive
    // carry of the segment after it; each segment publishes its own as
    // F + exp(A T) * that carry as soon as it knows it.  The aggregate passes
    // of all segments run in parallel and only this short step is chained,
    // always in segment order, so the result does not depend on timing.
    failed = __syncthreads_or(failed);
    tsum += __shfl_xor_sync(kFull, tsum, 16);  // both halves' steps
    int* my_flag = a.seg_flag + ((size_t)b * P.ntile + tile) * a.nseg + seg;
    float2 carry[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) carry[p] = make_float2(0.f, 0.f);
    if (!failed && seg < a.nseg - 1) {
      if (cta_wait_flag(my_flag + 1, P.spin_limit, wait_slot) == 0) {
        failed = true;
      } else {
        const float* src = a.segI + (((size_t)b * a.nseg + seg + 1) * Dm + (cvalid ? c : 0)) * kN;
        const float4 x0 = __ldcg(reinterpret_cast<const float4*>(src + q0));
        const float4 x1 = __ldcg(reinterpret_cast<const float4*>(src + (q0 ^ 4)));
        carry[0] = make_float2(x0.x, x0.y);
        carry[1] = make_float2(x0.z, x0.w);
        carry[2] = make_float2(x1.x, x1.y);
        carry[3] = make_float2(x1.z, x1.w);
      }
    }
    if (!failed && nagg) {  // publish the inclusive carry: F + exp(A T) carry
      const float2 t2 = dup2(tsum);
      float2 I[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 e = fmul2(A2[p], t2);
        I[p] = ffma2(make_float2(ex2(e.x), ex2(e.y)), carry[p], fa[p]);
      }
      if (cvalid) {
        float* dst = a.segI + (((size_t)b * a.nseg + seg) * Dm + c) * kN;
        *reinterpret_cast<float4*>(dst + q0) = make_float4(I[0].x, I[0].y, I[1].x, I[1].y);
        *reinterpret_cast<float4*>(dst + (q0 ^ 4)) = make_float4(I[2].x, I[2].y, I[3].x, I[3].y);
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) st_release_gpu(my_flag, kInclReady);
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) fa[p] = carry[p];  // the main pass starts from the true carry
  }

  for (int it = 0; it < nloc && !failed; ++it) {
    const int j = j1 - 1 - it;
    const int g = nagg + it;
    const int s = g % kBStages;
    const bool ok = mbar_wait_bounded(&bars[s], (g / kBStages) & 1);
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    const unsigned char* st = smem + s * S.stage;
    const T* su = reinterpret_cast<const T*>(st + S.offU) + cl;
    const T* sd = reinterpret_cast<const T*>(st + S.offDelta) + cl;
    const T* szo = reinterpret_cast<const T*>(st + S.offZo) + col;
    const T* sdo = reinterpret_cast<const T*>(st + S.offDo) + col;
    const T* suo = reinterpret_cast<const T*>(st + S.offUo) + col;
    const T* szs = reinterpret_cast<const T*>(st + S.offZs) + cl;
    const T* sds = reinterpret_cast<const T*>(st + S.offDs) + cl;
    const TBC* sB = reinterpret_cast<const TBC*>(st + S.offB);
    const TBC* sC = reinterpret_cast<const TBC*>(st + S.offC);
    float* red = sRed + (it & 1) * (kBWarps * kChunk * 32);

#pragma unroll 1
    for (int blk = 1; blk >= 0; --blk) {
      const int T0 = blk * kCk;
      const int ck = j * (kChunk / kCk) + blk;  // global 8-step block index
      // ---- per-step scalars: this lane evaluates step 2k + hs of each pair k
      // (own step) and receives the partner's step with one shuffle each.
      // (sgo: upstream gradient of the skip term in the scan frame; it differs
      // from dy only for the reference's reverse-skip frame; zgo: act'(z);
      // spo: d softplus / d delta)
      float dtv[kCk], dxv[kCk], dyv[kCk];
      float dto[kCk / 2], sgo[kCk / 2], zgo[kCk / 2], spo[kCk / 2];
#pragma unroll
      for (int k = 0; k < kCk / 2; ++k) {
        const int tl = T0 + 2 * k + hs;
        const bool valid = FAST || j * kChunk + tl < L;
        const float x = ld_f(su + tl * kBTile);
        const float dr = ld_f(sd + tl * kBTile) + bias;
        float sp = 1.f;
        float dt = softplus ? softplus_sig(dr, sp) : dr;
        dt = valid ? dt : 0.f;
        const float dx = valid ? dt * x : 0.f;
        const int row = rev ? kChunk - 1 - tl : tl;
        float g = ld_f(sdo + row * kBTile);
        float zg = 1.f;
        if (has_z) {
          float av;
          act_and_grad(ld_f(szo + row * kBTile), G, av, zg);
          g *= av;
        }
        const float dy = valid ? g : 0.f;
        float sg = dy;
        if (mirror) {
          sg = ld_f(sds + tl * kBTile);
          if (has_z) sg *= act_f(ld_f(szs + tl * kBTile), G);
          sg = valid ? sg : 0.f;
        }
        dto[k] = dt;
        sgo[k] = sg;
        zgo[k] = zg;
        spo[k] = sp;
        const float pdt = __shfl_xor_sync(kFull, dt, 16);
        const float pdx = __shfl_xor_sync(kFull, dx, 16);
        const float pdy = __shfl_xor_sync(kFull, dy, 16);
        dtv[2 * k] = own_odd ? pdt : dt;
        dtv[2 * k + 1] = own_odd ? dt : pdt;
        dxv[2 * k] = own_odd ? pdx : dx;
        dxv[2 * k + 1] = own_odd ? dx : pdx;
        dyv[2 * k] = own_odd ? pdy : dy;
        dyv[2 * k + 1] = own_odd ? dy : pdy;
      }
      // ---- restart state (the forward's checkpoint before this block)
      float2 h[4];
      if (ck > 0 && cvalid) {
        ld8q(st_b + (size_t)(ck - 1) * Dm * kN, q0, h);
      } else {
#pragma unroll
        for (int p = 0; p < 4; ++p) h[p] = make_float2(0.f, 0.f);
      }
      // ---- forward recompute: alpha, alpha*h to TMEM; y (for dz) and dC partials
      float yo[kCk / 2];  // y of this lane's own steps
#pragma unroll
      for (int u = 0; u < kCk; ++u) {
        const int tl = T0 + u;
        float2 Bq[4], Cq[4];
        ld8q(sB + tl * kN, q0, Bq);
        ld8q(sC + tl * kN, q0, Cq);
        const float2 dt2 = dup2(dtv[u]), dx2 = dup2(dxv[u]), dy2 = dup2(dyv[u]);
        float keep[16];
        float2 y2 = make_float2(0.f, 0.f), vc[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 e = fmul2(A2[p], dt2);
          const float2 al = make_float2(ex2(e.x), ex2(e.y));
          const float2 q = fmul2(al, h[p]);
          h[p] = ffma2(Bq[p], dx2, q);
          y2 = ffma2(Cq[p], h[p], y2);
          vc[p] = fmul2(dy2, h[p]);
          keep[2 * p] = al.x;
          keep[2 * p + 1] = al.y;
          keep[8 + 2 * p] = q.x;
          keep[8 + 2 * p + 1] = q.y;
        }
        tmem_st16_nc(trow + u * 16, keep);
        const float dc = reduce16ch(vc, b2, b1);
        if (red_writer) sts_nc(red + (warp * kChunk + tl) * 32 + kN + red_n, dc);
        float y = y2.x + y2.y;
        y += __shfl_xor_sync(kFull, y, 16);
        if (u & 1) yo[u >> 1] = own_odd ? y : yo[u >> 1];
        else yo[u >> 1] = y;
      }
      tmem_wait_st();

      // ---- adjoint sweep (TMEM reads double buffered one step ahead)
      float sbfo[kCk / 2], sawo[kCk / 2];
      uint32_t buf[2][16];
      tmem_ld16_nc(trow + (kCk - 1) * 16, buf[(kCk - 1) & 1]);
      tmem_wait_ld_regs(buf[(kCk - 1) & 1]);
#pragma unroll
      for (int u = kCk - 1; u >= 0; --u) {
        const int tl = T0 + u;
        if (u > 0) tmem_ld16_nc(trow + (u - 1) * 16, buf[(u - 1) & 1]);
        float2 Bq[4], Cq[4];
        ld8q(sB + tl * kN, q0, Bq);
        ld8q(sC + tl * kN, q0, Cq);
        const float2 dt2 = dup2(dtv[u]), dx2 = dup2(dxv[u]), dy2 = dup2(dyv[u]);
        float2 sAw = make_float2(0.f, 0.f), sBf = make_float2(0.f, 0.f), vb[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 al = make_float2(__uint_as_float(buf[u & 1][2 * p]), __uint_as_float(buf[u & 1][2 * p + 1]));
          const float2 q =
              make_float2(__uint_as_float(buf[u & 1][8 + 2 * p]), __uint_as_float(buf[u & 1][8 + 2 * p + 1]));
          const float2 f = ffma2(Cq[p], dy2, fa[p]);
          const float2 w = fmul2(f, q);
          dA[p] = ffma2(dt2, w, dA[p]);
          sAw = ffma2(A2[p], w, sAw);
          sBf = ffma2(Bq[p], f, sBf);
          vb[p] = fmul2(dx2, f);
          fa[p] = fmul2(f, al);
        }
        const float db = reduce16ch(vb, b2, b1);
        if (red_writer) sts_nc(red + (warp * kChunk + tl) * 32 + red_n, db);
        float sbf = sBf.x + sBf.y, saw = sAw.x + sAw.y;
        sbf += __shfl_xor_sync(kFull, sbf, 16);
        saw += __shfl_xor_sync(kFull, saw, 16);
        if (u & 1) {  // the sweep visits the odd step of a pair first
          sbfo[u >> 1] = sbf;
          sawo[u >> 1] = saw;
        } else {
          sbfo[u >> 1] = own_odd ? sbfo[u >> 1] : sbf;
          sawo[u >> 1] = own_odd ? sawo[u >> 1] : saw;
        }
        if (u > 0) tmem_wait_ld_regs(buf[(u - 1) & 1]);
      }

      // ---- epilogue of this lane's own steps: du, ddelta, dz and the skip
      // gradients (straight-line; steps past L and lanes past Dm hold zeros,
      // only the stores are predicated)
#pragma unroll
      for (int k = 0; k < kCk / 2; ++k) {
        const int tl = T0 + 2 * k + hs;
        const int t = j * kChunk + tl;
        const float x = ld_f(su + tl * kBTile);
        const float du = fmaf(Dsc, sgo[k], dto[k] * sbfo[k]);  // Dsc is 0 without a skip
        dD_acc = fmaf(sgo[k], x, dD_acc);
        const float g = fmaf(x, sbfo[k], sawo[k] * kLn2) * spo[k];  // d/d dt (A carried as A log2 e)
        db_acc += g;
        const bool st_ok = FAST || (t < L && cvalid);
        if (st_ok) {
          st_act(du_g + (size_t)t * Dm, du);
          st_act(dd_g + (size_t)t * Dm, g);
        }
        if (has_z) {  // dz needs the pre-gate output of the step
          const int row = rev ? kChunk - 1 - tl : tl;
          const int l = rev ? L - 1 - t : t;
          const float xs = mirror ? ld_f(suo + row * kBTile) : x;
          const float pre = fmaf(Dso, xs, yo[k]);  // Dso is 0 without a skip
          const float gz = ld_f(sdo + row * kBTile) * pre * zgo[k];
          if (st_ok) st_act(dz_g + (size_t)l * a.z_stride, gz);
        }
      }
    }

    __syncthreads();  // stage s consumed; red[] complete
    if (threadIdx.x == 0 && g + kBStages < ntot) {
      fence_proxy_async_smem();
      issue(g + kBStages);
    }
    if (threadIdx.x < kChunk * 8) {
      // sum the 8 warps' partials: thread -> (step, 4 consecutive outputs)
      const int tl = threadIdx.x >> 3, q4 = threadIdx.x & 7;
      const int t = j * kChunk + tl;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kBWarps; ++w) {
        const float4 p = *reinterpret_cast<const float4*>(red + (w * kChunk + tl) * 32 + q4 * 4);
        v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
      }
      if (t < L) {
        if constexpr (MC) {  // the sum over GPUs, done in the NVSwitch
          float* dst = (q4 < 4 ? a.dB_acc : a.dC_acc) + ((size_t)b * L + t) * a.acc_stride + (q4 & 3) * 4;
          multimem_red_add4(dst, v);
        } else {  // this tile's partial; finalize sums the tiles in order
          *reinterpret_cast<float4*>(a.bc_part + (((size_t)tile * P.batch + b) * L + t) * 32 + q4 * 4) = v;
        }
      }
    }
  }

  if constexpr (MC) __threadfence_system();  // dB / dC sums on other GPUs land before the kernel ends
  // release TMEM (every thread's accesses are complete)
  tmem_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, kBTmemCols);
  if (failed) {
    if (threadIdx.x == 0) report(a.status, kStatusTimeout);
    return;
  }
  dD_acc += __shfl_xor_sync(kFull, dD_acc, 16);
  db_acc += __shfl_xor_sync(kFull, db_acc, 16);
  if (cvalid) {
    const size_t r = (size_t)b * a.nseg + seg;
    float* dAp = a.dA_part + (r * Dm + c) * kN;
    *reinterpret_cast<float4*>(dAp + q0) = make_float4(dA[0].x, dA[0].y, dA[1].x, dA[1].y);
    *reinterpret_cast<float4*>(dAp + (q0 ^ 4)) = make_float4(dA[2].x, dA[2].y, dA[3].x, dA[3].y);
    if (hs == 0) {
      a.dD_part[r * Dm + c] = dD_acc;
      a.db_part[r * Dm + c] = db_acc;
    }
  }
}

}  // namespace ssm
