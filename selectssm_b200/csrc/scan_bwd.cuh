// Selective-scan backward kernel for B200 (sm_100a).
//
// Work decomposition
//   CTA   = one batch row b x 128 consecutive channels x one sequence segment;
//           4 warps, lane = channel, so every lane owns all 16 states of its
//           channel (packed f32x2 pairs).  Per-step scalars (softplus(dt),
//           dt*x, the gated upstream gradient) and the sums over states
//           (y, dx, ddt) are lane-local: no shuffles over states.
//   time  = TMA stages of 16 steps (u, delta, dout, z tiles of 128 ch x 16
//           steps; B and C tiles of 16 x 16), double buffered on mbarriers and
//           visited last to first; each stage is two 8-step blocks, last first.
//   block = restart from the state the forward saved before the block (plain
//           128-bit loads), recompute alpha_t = exp(A dt_t) and alpha_t h_{t-1}
//           for the 8 steps into tensor memory (TMEM: 8 steps x 32 values = 256
//           columns per lane, 2 CTAs per SM), then run the adjoint
//           f_t = alpha_{t+1} f_{t+1} + C_t dy_t backwards reading them back.
//   Leaf gradients (src/selectssm/ssmrecscan.py:150-161):
//     dx_t = dt_t sum_n f B_t,  dA += dt_t f alpha_t h_{t-1},  dB_t = sum_d dt_t x_t f,
//     dC_t = sum_d dy_t h_t,    ddt_t = sum_n f (A alpha_t h_{t-1} + B_t x_t).
//   dB / dC (sums over channels) use a shuffle reduce-scatter over the warp's
//   32 channels.  Lanes hold their 4 state quads in an order permuted by lane
//   bits 4 and 3 (A, B, C, the restart state and dA are read/written at the
//   permuted addresses), so the first two exchange stages need no selects.
//   The 4 warps' partials are summed in shared memory and stored as this
//   channel tile's partial; the finalize kernel sums the tiles in a fixed
//   order, so dB / dC are bit-reproducible.  dA/dD/d(delta_bias) are per-(batch row,
//   segment) partials summed in a fixed order by the finalize kernel.
//   The gate activation is a template parameter (fixed per launch) and the
//   per-step work holds no data- or flag-dependent branch (only stores are
//   predicated), so the compiler can schedule across the unrolled steps.
// Segments: ssm_bwd_agg_kernel runs segments 1..S-1 from a zero adjoint and
//   writes the adjoint carried out of each one's first step (one lane per
//   channel, 16 states; one state pair per lane evaluates its exponential on
//   the FMA pipe to relieve the MUFU unit); ssm_bwd_fold_kernel turns those
//   into the carry entering each segment.
#pragma once

#include "scan_kernels.cuh"

namespace ssm {

constexpr int kBTile = 128;                            // channels per backward CTA
constexpr int kBWarps = kBTile / 32;
constexpr int kBThreads = kBTile;
constexpr int kBStages = 2;
constexpr uint32_t kBTmemCols = kCk * 2 * kN;          // 8 steps x (16 alpha + 16 alpha*h)

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
  __host__ __device__ static uint32_t tx(int es, int esbc, bool has_z, bool mirror) {
    const int act = kChunk * kBTile * es, bc = kChunk * kN * esbc;
    return 3 * act + 2 * bc + (has_z ? act : 0) + (mirror ? (has_z ? 3 : 2) * act : 0);
  }
};

// Sum over the 32 channel-lanes of a warp of a lane's 16 per-state values
// (8 packed pairs).  Pair slot p holds states 4 (q ^ xq) + 2 (p & 1) + {0, 1},
// q = p >> 1, with xq = (lane bit 4) << 1 | (lane bit 3).  The result is the
// total for state 4 xq + 2 (lane bit 2) + (lane bit 1).
__device__ __forceinline__ float reduce32ch(const float2 (&v)[8], bool b2, bool b1) {
  float2 r[4];
#pragma unroll
  for (int p = 0; p < 4; ++p)  // lane bit 4: keep quads 0,1, receive the partner's quads 2,3
    r[p] = fadd2(v[p], make_float2(__shfl_xor_sync(kFull, v[p + 4].x, 16), __shfl_xor_sync(kFull, v[p + 4].y, 16)));
#pragma unroll
  for (int p = 0; p < 2; ++p)  // lane bit 3: keep quad 0
    r[p] = fadd2(r[p], make_float2(__shfl_xor_sync(kFull, r[p + 2].x, 8), __shfl_xor_sync(kFull, r[p + 2].y, 8)));
  // lane bit 2: keep one pair of the quad
  const float2 kp = b2 ? r[1] : r[0], sd = b2 ? r[0] : r[1];
  const float2 s = fadd2(kp, make_float2(__shfl_xor_sync(kFull, sd.x, 4), __shfl_xor_sync(kFull, sd.y, 4)));
  // lane bit 1: keep one element of the pair
  float q = (b1 ? s.y : s.x) + __shfl_xor_sync(kFull, b1 ? s.x : s.y, 2);
  q += __shfl_xor_sync(kFull, q, 1);  // lane bit 0: both lanes keep the total
  return q;
}

// 16 per-state values at permuted quad addresses -> 8 pairs
template <typename TB>
__device__ __forceinline__ void ld16q(const TB* row, int xq, float2 (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = ld4(row + 4 * (q ^ xq));
    v[2 * q] = make_float2(f.x, f.y);
    v[2 * q + 1] = make_float2(f.z, f.w);
  }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// G: the gate activation (an ssm_act code), fixed per launch so the step loops
// hold no branch on it.
// MC: dB / dC partial sums go to NVLink multicast addresses (cross-GPU sum);
// a template parameter so the single-GPU instance carries no trace of it.
template <typename T, typename TBC, int G, bool MC = false>
__global__ void __launch_bounds__(kBThreads, 2) ssm_bwd_kernel(const __grid_constant__ BwdLaunch P) {
  const BwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = blockIdx.z % P.zdiv;
  extern __shared__ __align__(1024) unsigned char smem[];

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kBTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = threadIdx.x;  // channel within the tile
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
  const int nck = (L + kCk - 1) / kCk;
  const int j1 = min(nblk, (seg + 1) * a.seg_chunks);
  const int nloc = j1 - seg * a.seg_chunks;
  const bool cvalid = c < Dm;
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
  const uint32_t trow = tbase + ((uint32_t)(warp * 32) << 16);  // this warp's lane quarter

  const uint32_t tx = BwdLayout::tx(sizeof(T), sizeof(TBC), has_z, mirror);
  auto issue = [&](int it) {  // it-th load is chunk j1-1-it (last first)
    const int j = j1 - 1 - it;
    unsigned char* st = smem + (it % kBStages) * S.stage;
    uint64_t* bar = &bars[it % kBStages];
    const int t0 = j * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, tx);
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
  };
  if (threadIdx.x == 0) {
    const int npre = nloc < kBStages ? nloc : kBStages;
    for (int it = 0; it < npre; ++it) issue(it);
  }

  // state permutation (see reduce32ch)
  const int xq = (((lane >> 4) & 1) << 1) | ((lane >> 3) & 1);
  const bool b2 = ((lane >> 2) & 1) != 0, b1 = ((lane >> 1) & 1) != 0;
  const int red_n = 4 * xq + (b2 ? 2 : 0) + (b1 ? 1 : 0);
  const bool red_writer = (lane & 1) == 0;
  // A (pairs at the permuted quad addresses) is re-read from L1 at each use
  // rather than held in 16 registers.
  const float* Arow = a.A + (size_t)(cvalid ? c : 0) * kN;
  auto An_at = [&](int p) {
    return __ldg(reinterpret_cast<const float2*>(Arow + 4 * ((p >> 1) ^ xq) + 2 * (p & 1)));
  };
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  const float Dsc = (has_D && cvalid) ? a.D[c] : 0.f;                  // skip weight, scan channel
  const float Dso = (has_D && cvalid) ? a.D[aligned ? c : co] : 0.f;   // skip weight in the pre-gate value
  float2 fa[8], dA[8];  // f_{t+1} alpha_{t+1} carried backwards; dA accumulators
#pragma unroll
  for (int p = 0; p < 8; ++p) fa[p] = dA[p] = make_float2(0.f, 0.f);
  if (a.nseg > 1 && cvalid)  // adjoint entering this segment from the later ones
    ld16q(a.segF + (((size_t)b * a.nseg + seg) * Dm + c) * kN, xq, fa);
  float dD_acc = 0.f, db_acc = 0.f;
  T* du_g = reinterpret_cast<T*>(a.du) + (size_t)b * L * Dm + c;
  T* dd_g = reinterpret_cast<T*>(a.ddelta) + (size_t)b * L * Dm + c;
  T* dz_g = reinterpret_cast<T*>(a.dz) + (size_t)b * L * a.z_stride + co;
  const float* st_b = a.states + ((size_t)b * nck * Dm + (cvalid ? c : 0)) * kN;
  bool failed = false;

  for (int it = 0; it < nloc; ++it) {
    const int j = j1 - 1 - it;
    const int s = it % kBStages;
    const bool ok = mbar_wait_bounded(&bars[s], (it / kBStages) & 1);
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
      // ---- per-step scalars of the block (own channel)
      // (sgv: upstream gradient of the skip term in the scan frame; it differs
      // from dyv only for the reference's reverse-skip frame)
      // (zgv: act'(z) of the step, for dz; spv: d softplus / d delta, for ddelta)
      float dtv[kCk], dxv[kCk], dyv[kCk], sgv[kCk], zgv[kCk], spv[kCk];
#pragma unroll
      for (int u = 0; u < kCk; ++u) {
        const int tl = T0 + u;
        const bool valid = j * kChunk + tl < L;
        const float x = ld_f(su + tl * kBTile);
        const float dr = ld_f(sd + tl * kBTile) + bias;
        spv[u] = 1.f;
        const float dt = softplus ? softplus_sig(dr, spv[u]) : dr;
        dtv[u] = valid ? dt : 0.f;
        dxv[u] = valid ? dt * x : 0.f;
        const int row = rev ? kChunk - 1 - tl : tl;
        float g = ld_f(sdo + row * kBTile);
        zgv[u] = 1.f;
        if (has_z) {
          float av;
          act_and_grad(ld_f(szo + row * kBTile), G, av, zgv[u]);
          g *= av;
        }
        dyv[u] = valid ? g : 0.f;
        sgv[u] = dyv[u];
      }
      if (mirror) {
#pragma unroll
        for (int u = 0; u < kCk; ++u) {
          const int tl = T0 + u;
          float sg = ld_f(sds + tl * kBTile);
          if (has_z) sg *= act_f(ld_f(szs + tl * kBTile), G);
          sgv[u] = j * kChunk + tl < L ? sg : 0.f;
        }
      }
      // ---- restart state (the forward's checkpoint before this block)
      float2 h[8];
      if (ck > 0 && cvalid) {
        ld16q(st_b + (size_t)(ck - 1) * Dm * kN, xq, h);
      } else {
#pragma unroll
        for (int p = 0; p < 8; ++p) h[p] = make_float2(0.f, 0.f);
      }
      // ---- forward recompute: alpha, alpha*h to TMEM; y (for dz) and dC partials
#pragma unroll
      for (int u = 0; u < kCk; ++u) {
        const int tl = T0 + u;
        float2 Bq[8], Cq[8];
        ld16q(sB + tl * kN, xq, Bq);
        ld16q(sC + tl * kN, xq, Cq);
        const float2 dt2 = dup2(dtv[u] * kLog2e), dx2 = dup2(dxv[u]), dy2 = dup2(dyv[u]);
        float keep[32];
        float2 y2 = make_float2(0.f, 0.f), vc[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const float2 e = fmul2(An_at(p), dt2);
          const float2 al = make_float2(ex2(e.x), ex2(e.y));
          const float2 q = fmul2(al, h[p]);
          h[p] = ffma2(Bq[p], dx2, q);
          y2 = ffma2(Cq[p], h[p], y2);
          vc[p] = fmul2(dy2, h[p]);
          keep[2 * p] = al.x;
          keep[2 * p + 1] = al.y;
          keep[16 + 2 * p] = q.x;
          keep[16 + 2 * p + 1] = q.y;
        }
        tmem_st32(trow + u * 32, keep);
        const float dc = reduce32ch(vc, b2, b1);
        if (red_writer) red[(warp * kChunk + tl) * 32 + kN + red_n] = dc;
        // dz needs the pre-gate output of this step
        if (has_z) {  // straight-line; only the store is predicated
          const int t = j * kChunk + tl;
          const int row = rev ? kChunk - 1 - tl : tl;
          const int l = rev ? L - 1 - t : t;
          const float xs = ld_f(mirror ? suo + row * kBTile : su + tl * kBTile);
          const float pre = fmaf(Dso, xs, y2.x + y2.y);  // Dso is 0 without a skip
          const float g = ld_f(sdo + row * kBTile) * pre * zgv[u];
          if (t < L && cvalid) st_act(dz_g + (size_t)l * a.z_stride, g);
        }
      }
      tmem_wait_st();

      // ---- adjoint sweep (TMEM reads double buffered one step ahead)
      uint32_t buf[2][32];
      tmem_ld32(trow + (kCk - 1) * 32, buf[(kCk - 1) & 1]);
      tmem_wait_ld();
#pragma unroll
      for (int u = kCk - 1; u >= 0; --u) {
        const int tl = T0 + u;
        if (u > 0) tmem_ld32(trow + (u - 1) * 32, buf[(u - 1) & 1]);
        float2 Bq[8], Cq[8];
        ld16q(sB + tl * kN, xq, Bq);
        ld16q(sC + tl * kN, xq, Cq);
        const float2 dt2 = dup2(dtv[u]), dx2 = dup2(dxv[u]), dy2 = dup2(dyv[u]);
        float2 sAw = make_float2(0.f, 0.f), sBf = make_float2(0.f, 0.f), vb[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const float2 al = make_float2(__uint_as_float(buf[u & 1][2 * p]), __uint_as_float(buf[u & 1][2 * p + 1]));
          const float2 q =
              make_float2(__uint_as_float(buf[u & 1][16 + 2 * p]), __uint_as_float(buf[u & 1][16 + 2 * p + 1]));
          const float2 f = ffma2(Cq[p], dy2, fa[p]);
          const float2 w = fmul2(f, q);
          dA[p] = ffma2(dt2, w, dA[p]);
          sAw = ffma2(An_at(p), w, sAw);
          sBf = ffma2(Bq[p], f, sBf);
          vb[p] = fmul2(dx2, f);
          fa[p] = fmul2(f, al);
        }
        const float sbf = sBf.x + sBf.y, saw = sAw.x + sAw.y;
        const float db = reduce32ch(vb, b2, b1);
        if (red_writer) red[(warp * kChunk + tl) * 32 + red_n] = db;
        // du, ddelta and the skip gradients of this step
        // straight-line (steps past L and lanes past Dm hold zeros); only the
        // stores are predicated
        const int t = j * kChunk + tl;
        const float x = ld_f(su + tl * kBTile);
        const float du = fmaf(Dsc, sgv[u], dtv[u] * sbf);  // Dsc is 0 without a skip
        dD_acc = fmaf(sgv[u], x, dD_acc);
        float g = fmaf(x, sbf, saw);  // d/d dt
        g *= spv[u];
        db_acc += g;
        if (t < L && cvalid) {
          st_act(du_g + (size_t)t * Dm, du);
          st_act(dd_g + (size_t)t * Dm, g);
        }
        if (u > 0) tmem_wait_ld();
      }
    }

    __syncthreads();  // stage s consumed; red[] complete
    if (threadIdx.x == 0 && it + kBStages < nloc) {
      fence_proxy_async_smem();
      issue(it + kBStages);
    }
    {
      // sum the 4 warps' partials: thread -> (step, 4 consecutive outputs)
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
          *reinterpret_cast<float4*>(a.bc_part + (((size_t)blockIdx.x * gridDim.y + b) * L + t) * 32 + q4 * 4) = v;
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
  if (cvalid) {
    const size_t r = (size_t)b * a.nseg + seg;
    float* dAp = a.dA_part + (r * Dm + c) * kN;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<float4*>(dAp + 4 * (q ^ xq)) =
          make_float4(dA[2 * q].x, dA[2 * q].y, dA[2 * q + 1].x, dA[2 * q + 1].y);
    a.dD_part[r * Dm + c] = dD_acc;
    a.db_part[r * Dm + c] = db_acc;
  }
}

// Backward segment pre-pass: for segment s >= 1 runs the adjoint recurrence
// f_t = C_t dy_t + f_{t+1} alpha_{t+1} over the segment from a zero carry and
// writes the carry leaving its first step (f alpha, natural state order) and
// the segment's sum of dt.  Reads delta, C, dout and z only.
// State pairs per lane whose exponential the pre-pass evaluates on the FMA
// pipe (ex2_poly2): the pre-pass is otherwise bound by the MUFU unit.
constexpr int kAggEmu = 1;

struct BwdAggLayout {
  int offDelta, offDo, offZo, offC, stage, offBars, bytes;
  __host__ __device__ BwdAggLayout(int es, int esbc, bool has_z) {
    const int act = kChunk * kBTile * es, bc = kChunk * kN * esbc;
    int o = 0;
    offDelta = o; o += act;
    offDo = o; o += act;
    offZo = o; if (has_z) o += act;
    offC = o; o += bc;
    stage = (o + 127) & ~127;
    offBars = stage * kBStages;
    bytes = offBars + 8 * kBStages;
  }
};

template <typename T, typename TBC, int G>
__global__ void __launch_bounds__(kBThreads, 4) ssm_bwd_agg_kernel(const __grid_constant__ BwdLaunch P) {
  const BwdDir& a = P.dir[blockIdx.z / P.zdiv];
  const int seg = 1 + blockIdx.z % P.zdiv;  // segments 1 .. nseg-1
  extern __shared__ __align__(1024) unsigned char smem[];
  const int b = blockIdx.y;
  const int c0 = blockIdx.x * kBTile;
  const int cl = threadIdx.x;
  const int c = c0 + cl;
  const int L = a.L, Dm = a.Dm;
  if (c0 >= Dm) return;
  const bool rev = (a.flags & SSM_REVERSE) != 0;
  const bool comp = rev && (a.flags & SSM_COMPLEMENT);
  const bool softplus = (a.flags & SSM_DELTA_SOFTPLUS) != 0;
  const bool has_z = a.has_z != 0;
  const int nblk = (L + kChunk - 1) / kChunk;
  const int j1 = min(nblk, (seg + 1) * a.seg_chunks);
  const int nloc = j1 - seg * a.seg_chunks;
  const bool cvalid = c < Dm;
  const int oc0 = comp ? Dm - kBTile - c0 : c0;
  const int col = comp ? kBTile - 1 - cl : cl;
  const BwdAggLayout S(sizeof(T), sizeof(TBC), has_z);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.offBars);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t tx = (2 + (has_z ? 1 : 0)) * kChunk * kBTile * (int)sizeof(T) + kChunk * kN * (int)sizeof(TBC);
  auto issue = [&](int it) {
    const int j = j1 - 1 - it;
    unsigned char* st = smem + (it % kBStages) * S.stage;
    uint64_t* bar = &bars[it % kBStages];
    const int t0 = j * kChunk;
    const int ot0 = rev ? L - kChunk - t0 : t0;
    mbar_arrive_expect_tx(bar, tx);
    tma_load_3d(st + S.offDelta, &a.tm_delta, bar, c0, t0, b);
    tma_load_3d(st + S.offC, &a.tm_C, bar, 0, t0, b);
    tma_load_3d(st + S.offDo, &a.tm_dout, bar, oc0, ot0, b);
    if (has_z) tma_load_3d(st + S.offZo, &a.tm_z, bar, oc0, ot0, b);
  };
  if (threadIdx.x == 0) {
    const int npre = nloc < kBStages ? nloc : kBStages;
    for (int it = 0; it < npre; ++it) issue(it);
  }
  float2 A2[8];
  {
    const float* Ar = a.A + (size_t)(cvalid ? c : 0) * kN;
#pragma unroll
    for (int p = 0; p < 8; ++p)
      A2[p] = cvalid ? make_float2(Ar[2 * p] * kLog2e, Ar[2 * p + 1] * kLog2e) : make_float2(0.f, 0.f);
  }
  const float bias = (a.bias && cvalid) ? a.bias[c] : 0.f;
  float2 fa[8];
#pragma unroll
  for (int p = 0; p < 8; ++p) fa[p] = make_float2(0.f, 0.f);
  float tsum = 0.f;
  for (int it = 0; it < nloc; ++it) {
    const int j = j1 - 1 - it;
    const int s = it % kBStages;
    const bool ok = mbar_wait_bounded(&bars[s], (it / kBStages) & 1);
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) report(a.status, kStatusTimeout);
      return;
    }
    const unsigned char* st = smem + s * S.stage;
    const T* sd = reinterpret_cast<const T*>(st + S.offDelta) + cl;
    const T* sdo = reinterpret_cast<const T*>(st + S.offDo) + col;
    const T* szo = reinterpret_cast<const T*>(st + S.offZo) + col;
    const TBC* sC = reinterpret_cast<const TBC*>(st + S.offC);
#pragma unroll
    for (int tl = kChunk - 1; tl >= 0; --tl) {
      const bool valid = j * kChunk + tl < L;
      const float dr = ld_f(sd + tl * kBTile) + bias;
      float dt = softplus ? softplus_f(dr) : dr;
      dt = valid ? dt : 0.f;
      tsum += dt;
      const int row = rev ? kChunk - 1 - tl : tl;
      float g = ld_f(sdo + row * kBTile);
      if (has_z) g *= act_f(ld_f(szo + row * kBTile), G);
      const float2 dy2 = dup2(valid ? g : 0.f), dt2 = dup2(dt);
      float2 Cq[8];
      ld16q(sC + tl * kN, 0, Cq);
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const float2 e = fmul2(A2[p], dt2);
        const float2 al = p < kAggEmu ? ex2_poly2(e) : make_float2(ex2(e.x), ex2(e.y));
        fa[p] = fmul2(ffma2(Cq[p], dy2, fa[p]), al);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && it + kBStages < nloc) {
      fence_proxy_async_smem();
      issue(it + kBStages);
    }
  }
  if (cvalid) {
    const size_t r = (size_t)b * a.nseg + seg;
    float4* F = reinterpret_cast<float4*>(a.segF + (r * Dm + c) * kN);
#pragma unroll
    for (int q = 0; q < 4; ++q) F[q] = make_float4(fa[2 * q].x, fa[2 * q].y, fa[2 * q + 1].x, fa[2 * q + 1].y);
    a.segT[r * Dm + c] = tsum;
  }
}

}  // namespace ssm
