// C-ABI entry points for the selective scan (forward, backward, bidirectional),
// their argument checks, TMA descriptor set-up and launch sequences.
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "scan_bwd.cuh"
#include "scan_fwd.cuh"
#include "scan_fwd_lane.cuh"

namespace ssm {

// Detail of the most recent SSM_ERR_LAUNCH on this host thread (diagnostics only).
thread_local char g_last_error[256] = "";
std::atomic<unsigned long long> g_launches{0};

void note_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int launch_error(const char* where, cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, cudaGetErrorString(e));
  return SSM_ERR_LAUNCH;
}
// Makes the device that owns `ptr` current for this library's runtime on the
// calling thread (and its primary context current for driver calls such as
// cuTensorMapEncodeTiled).  Callers may run on any host thread (e.g. an autograd
// worker) and any device.
int bind_device(const void* ptr) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) return launch_error("cudaPointerGetAttributes", e);
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) {
    snprintf(g_last_error, sizeof(g_last_error), "pointer %p is not device memory", ptr);
    return SSM_ERR_LAUNCH;
  }
  e = cudaSetDevice(a.device);
  if (e != cudaSuccess) return launch_error("cudaSetDevice", e);
  return SSM_OK;
}

#define SSM_CUDA_CHECK(call, where)        \
  do {                                     \
    cudaError_t e_ = (call);               \
    if (e_ != cudaSuccess) return launch_error(where, e_); \
  } while (0)

// ---------------------------------------------------------------- small kernels
// Widens the bf16 rows of B and C (16 elements, row stride `stride` elements)
// to dense float32 rows, one 16-byte load (8 elements) per thread and tensor.
// The scan kernels read every B / C element once per channel, so converting
// once per call here is cheaper than converting in every lane.
__global__ void widen_bc_kernel(const __nv_bfloat16* __restrict__ Bm, const __nv_bfloat16* __restrict__ Cm,
                                int64_t rows, int64_t stride, float* __restrict__ Bw, float* __restrict__ Cw) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * 2) return;
  const int64_t r = i >> 1, h = (i & 1) * 8;
  const __nv_bfloat16* src[2] = {Bm, Cm};
  float* dst[2] = {Bw, Cw};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint4 v = *reinterpret_cast<const uint4*>(src[k] + r * stride + h);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = __uint_as_float(w[j] << 16);
      f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
    float4* o = reinterpret_cast<float4*>(dst[k] + r * kN + h);
    o[0] = make_float4(f[0], f[1], f[2], f[3]);
    o[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

template <typename TBC>
__global__ void finalize_kernel(FinalizeDir f) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nDN = (int64_t)f.Dm * kN;
  if (i < nDN) {  // dA: sum over batch rows in order
    float s = 0.f;
    for (int b = 0; b < f.prows; ++b) s += f.dA_part[(int64_t)b * nDN + i];
    f.dA[i] = s;
  }
  if (i < f.Dm) {
    if (f.dD) {
      float s = 0.f;
      for (int b = 0; b < f.prows; ++b) s += f.dD_part[(int64_t)b * f.Dm + i];
      f.dD[i] = s;
    }
    if (f.dbias) {
      float s = 0.f;
      for (int b = 0; b < f.prows; ++b) s += f.db_part[(int64_t)b * f.Dm + i];
      f.dbias[i] = s;
    }
  }
  if (f.bc_part) {  // dB | dC: sum the channel tiles' partials in tile order, 4 states per thread
    const int64_t rows = (int64_t)f.batch * f.L;
    const float4* P = reinterpret_cast<const float4*>(f.bc_part);
    for (int64_t e = i; e < rows * 8; e += (int64_t)gridDim.x * blockDim.x) {
      float4 v = P[e];
      for (int k = 1; k < f.ntile; ++k) {
        const float4 w = P[(int64_t)k * rows * 8 + e];
        v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
      }
      const int64_t r = e >> 3;
      const int q = (int)(e & 7);
      TBC* dst = reinterpret_cast<TBC*>(q < 4 ? f.dB : f.dC) + r * f.bc_stride + (q & 3) * 4;
      dst[0] = Cvt<TBC>::from_f(v.x);
      dst[1] = Cvt<TBC>::from_f(v.y);
      dst[2] = Cvt<TBC>::from_f(v.z);
      dst[3] = Cvt<TBC>::from_f(v.w);
    }
  }
}

// ---------------------------------------------------------------- TMA descriptors
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {  // resolved once, read-only afterwards
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D tiled map over (d0 innermost, d1, d2) with row strides in bytes.
static bool make_map(CUtensorMap* m, const void* base, bool bf16, uint64_t d0, uint64_t d1, uint64_t d2,
                     uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled not available from the driver");
    return false;
  }
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                        const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    snprintf(g_last_error, sizeof(g_last_error),
             "cuTensorMapEncodeTiled error %d: base %p dims {%llu,%llu,%llu} strides {%llu,%llu} box {%u,%u}",
             (int)r, base, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
             (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes, box0, box1);
  return r == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- validation
static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Geo {
  int B, L, Dm, nblk;
  int es, esbc;  // element sizes
  bool bf16, bcbf16;
  int64_t zs, os, bs;  // row strides in elements
  int ndir;             // directions in one launch (2 for the *_bidir calls)
};

static int check_common(const ssm_params_t* p, Geo* g) {
  if (!p) return SSM_ERR_NULL;
  if (p->batch < 0 || p->seqlen < 0 || p->dim < 0) return SSM_ERR_SHAPE;
  if (p->dstate != kN) return SSM_ERR_SHAPE;
  if (p->batch > 65535) return SSM_ERR_SHAPE;
  if ((p->dtype != SSM_F32 && p->dtype != SSM_BF16) || (p->bc_dtype != SSM_F32 && p->bc_dtype != SSM_BF16))
    return SSM_ERR_DTYPE;
  if (p->gate_act < SSM_ACT_NONE || p->gate_act > SSM_ACT_RELU) return SSM_ERR_SHAPE;
  g->ndir = 1;
  g->B = p->batch;
  g->L = p->seqlen;
  g->Dm = p->dim;
  g->nblk = (p->seqlen + kChunk - 1) / kChunk;
  g->bf16 = p->dtype == SSM_BF16;
  g->bcbf16 = p->bc_dtype == SSM_BF16;
  g->es = g->bf16 ? 2 : 4;
  g->esbc = g->bcbf16 ? 2 : 4;
  g->zs = p->z_stride ? p->z_stride : p->dim;
  g->os = p->out_stride ? p->out_stride : p->dim;
  g->bs = p->bc_stride ? p->bc_stride : kN;
  if (g->zs < p->dim || g->os < p->dim || g->bs < kN) return SSM_ERR_SHAPE;
  // TMA: channel tiles (incl. the mirrored complement tile) start on 16-byte
  // boundaries, and every row stride is a multiple of 16 bytes.
  if (((int64_t)p->dim * g->es) % 16 || (g->zs * g->es) % 16 || (g->os * g->es) % 16 ||
      (g->bs * g->esbc) % 16)
    return SSM_ERR_ALIGN;
  return SSM_OK;
}

// inputs shared by the forward and the backward
static int check_inputs(const ssm_params_t* p, Geo* g) {
  int st = check_common(p, g);
  if (st) return st;
  if ((int64_t)g->B * g->L * g->Dm == 0) return SSM_OK;
  if (!p->u || !p->delta || !p->A || !p->Bm || !p->Cm || !p->states) return SSM_ERR_NULL;
  if (!aligned16(p->u) || !aligned16(p->delta) || !aligned16(p->Bm) || !aligned16(p->Cm) ||
      !aligned16(p->states) || !aligned16(p->A) || (p->z && !aligned16(p->z)))
    return SSM_ERR_ALIGN;
  return SSM_OK;
}

static int check_fwd(const ssm_params_t* p, Geo* g) {
  int st = check_inputs(p, g);
  if (st) return st;
  if ((int64_t)g->B * g->L * g->Dm != 0 && !p->out) return SSM_ERR_NULL;
  return SSM_OK;
}

static int check_bwd(const ssm_params_t* p, Geo* g) {
  int st = check_inputs(p, g);
  if (st) return st;
  if (!p->dA || (p->D && !p->dD) || (p->delta_bias && !p->ddelta_bias)) return SSM_ERR_NULL;
  if ((int64_t)g->B * g->L * g->Dm == 0) return SSM_OK;
  if (!p->dout || !p->du || !p->ddelta || !p->dB || !p->dC || (p->z && !p->dz)) return SSM_ERR_NULL;
  if (!aligned16(p->dout) || !aligned16(p->dB) || !aligned16(p->dC)) return SSM_ERR_ALIGN;
  return SSM_OK;
}

static size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Sequence segments.  A (batch row, channel tile) is one chain of steps; with
// few chains the sequence is cut into segments that run as separate CTAs of
// one launch: a segment that a later one depends on first runs an aggregate
// pass over its own steps and publishes it, and every segment folds the
// published values before it (decoupled lookback).  The segment count
// minimises a model of the run time in units of "one CTA processing one
// 16-step stage", from the duration of one CTA (its main pass, its aggregate
// pass at relative cost r, a fixed cost) and the number of resident CTAs:
// the total work spread evenly plus one CTA's duration (the tail).  The
// backward instead follows a fill rule fitted to measurements.  The resident counts are fixed here (not
// queried), so workspace sizes stay a function of the shapes alone.
struct Seg {
  int nseg, seg_chunks;
};
struct SegPolicy {
  int max_seg;      // segment cap
  bool per_launch;  // count the chains of both directions of a bidirectional launch
  int tile;         // channels per CTA
  long slots;       // resident CTAs of the main kernel on the GPU
  long agg_slots;   // resident CTAs of the pre-pass
  double agg_cost;  // pre-pass cost of one stage relative to the main kernel's
  bool single_pass; // pre-pass inside the main launch (decoupled lookback)
  double cta_cost;  // fixed cost of one CTA in stages (set-up, pipeline fill, lookback)
  bool fill_rule;   // pick by the fill rule below instead of the cost model
};
constexpr int kSMs = 148;
// The forward's CTAs are small and latency bound, so its resident-CTA count is
// an effective size fitted to measurements (batch 8 runs best unsegmented with
// 384 CTAs) rather than an occupancy limit.  Its choice holds per direction: a
// bidirectional launch (B=2, L=131072, 512 channels) ran faster with the
// per-direction choice than with one that counts both directions' chains.
#ifndef SSM_FWD_SLOTS
#define SSM_FWD_SLOTS 384
#endif
constexpr SegPolicy kFwdSeg{256, false, kTileCh, SSM_FWD_SLOTS, SSM_FWD_SLOTS, 0.8, true, 8.0, false};
constexpr SegPolicy kBwdSeg{256, true, kBTile, 2L * kSMs, 2L * kSMs, 0.2, true, 2.0, true};  // fill rule

static Seg choose_segments(const Geo& g, SegPolicy pol) {
  const int nblk = (g.L + kChunk - 1) / kChunk;
  if (nblk == 0) return {1, 1};
#ifdef SSM_EXP_ENV
  if (const char* e = getenv(pol.tile == kBTile ? "SSM_BWD_NSEG" : "SSM_FWD_NSEG")) {
    int n = atoi(e);
    if (n < 1) n = 1;
    if (n > nblk) n = nblk;
    const int sc = (nblk + n - 1) / n;
    return {(nblk + sc - 1) / sc, sc};
  }
#endif
  // both directions of a bidirectional call share the launch
  const long chains = (long)((g.Dm + pol.tile - 1) / pol.tile) * g.B * (pol.per_launch ? g.ndir : 1);
  if (chains <= 0) return {1, nblk};
  int max_seg = nblk / 4;  // at least 4 stages (64 steps) per segment
  if (max_seg < 1) max_seg = 1;
  if (max_seg > pol.max_seg) max_seg = pol.max_seg;
  if (pol.fill_rule) {
    // Measured on the backward (batches 8 to 64 of 1536 channels): with at
    // least two waves of chains the sequence is not cut; otherwise as many
    // segments as fit in two waves of CTAs (four when that is fewer than two
    // segments), and at least one per 64 stages (1024 steps), since shorter
    // CTAs balance better across the SMs than a few long ones.
    if (chains >= 2 * pol.slots) return {1, nblk};
    long n = 2 * pol.slots / chains;
    if (n < 2) n = 4 * pol.slots / chains;
    n = std::max<long>(n, nblk / 64);
    if (n > max_seg) n = max_seg;
    const int sc = (nblk + (int)n - 1) / (int)n;
    return {(nblk + sc - 1) / sc, sc};
  }
  double best = 0.0;
  Seg pick{1, nblk};
  for (int n = 1; n <= max_seg; ++n) {
    const int seg_chunks = (nblk + n - 1) / n;
    const int nseg = (nblk + seg_chunks - 1) / seg_chunks;
    if (nseg != n) continue;  // the same split as a smaller n
    double cost;
    if (pol.single_pass) {  // CTAs that each run an aggregate pass and a main pass
      const double per_cta = seg_chunks * (1.0 + (nseg > 1 ? pol.agg_cost : 0.0)) + pol.cta_cost;
      const double work = (double)chains * (seg_chunks * (nseg + pol.agg_cost * (nseg - 1)) + pol.cta_cost * nseg);
      cost = work / pol.slots + per_cta;
    } else {
      const long waves = (chains * nseg + pol.slots - 1) / pol.slots;
      const long agg_waves = (chains * (nseg - 1) + pol.agg_slots - 1) / pol.agg_slots;
      cost = (double)waves * seg_chunks + pol.agg_cost * (double)agg_waves * seg_chunks + 0.25 * nseg;
    }
    if (n == 1 || cost < best) {
      best = cost;
      pick = {nseg, seg_chunks};
    }
  }
  return pick;
}

// float32 copies of bf16 B and C rows (see widen_bc_kernel)
static size_t wide_bc_bytes(const Geo& g) {
  return g.bcbf16 ? 2 * round256((size_t)g.B * g.L * kN * 4) : 0;
}

// lookback flags of one direction: a 16-byte word (the launch's CTA ticket,
// used in the first direction's region) then one int per (row, tile, segment)
static size_t flag_bytes(const Geo& g, int nseg, int tile) {
  return round256(16 + (size_t)g.B * ((g.Dm + tile - 1) / tile) * nseg * 4);
}

// segI, flags
static size_t fwd_seg_bytes(const Geo& g) {
  const Seg sg = choose_segments(g, kFwdSeg);
  if (sg.nseg <= 1) return 0;
  const size_t rows = (size_t)g.B * sg.nseg * g.Dm;
  return round256(rows * kN * 4) + flag_bytes(g, sg.nseg, kTileCh);
}

static size_t fwd_ws_bytes(const Geo& g) { return fwd_seg_bytes(g) + wide_bc_bytes(g); }

// per-channel-tile dB | dC partials: (tiles, B, L, 32) float32
static size_t bc_part_bytes(const Geo& g) {
  return round256((size_t)((g.Dm + kBTile - 1) / kBTile) * g.B * g.L * 2 * kN * 4);
}

static size_t bwd_flag_bytes(const Geo& g, int nseg) { return flag_bytes(g, nseg, kBTile); }

static size_t bwd_ws_bytes(const Geo& g, bool multicast = false) {
  const Seg sg = choose_segments(g, kBwdSeg);
  const size_t rows = (size_t)g.B * sg.nseg * g.Dm;
  size_t n = round256(rows * kN * 4) + 2 * round256(rows * 4);
  if (sg.nseg > 1)  // segI, flags
    n += round256(rows * kN * 4) + bwd_flag_bytes(g, sg.nseg);
  if (!multicast) n += bc_part_bytes(g);  // the multicast form sums dB / dC in the caller's buffer
  return n + wide_bc_bytes(g);
}

// The segment count depends on whether the call is bidirectional, which a
// single parameter set does not say: size for both.
static size_t ws_bytes(const Geo& g) {
  size_t n = 0;
  for (int nd = 1; nd <= 2; ++nd) {
    Geo h = g;
    h.ndir = nd;
    n = std::max({n, fwd_ws_bytes(h), bwd_ws_bytes(h)});
  }
  return n;
}

static int launch_widen_bc(const ssm_params_t* p, const Geo& g, float* Bw, float* Cw, cudaStream_t s) {
  const int64_t rows = (int64_t)g.B * g.L;
  const int threads = 256;
  const unsigned blocks = (unsigned)((rows * 2 + threads - 1) / threads);
  widen_bc_kernel<<<blocks, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(p->Bm),
                                              static_cast<const __nv_bfloat16*>(p->Cm), rows, g.bs, Bw, Cw);
  note_launches(1);
  SSM_CUDA_CHECK(cudaGetLastError(), "launch widen_bc_kernel");
  return SSM_OK;
}

// B / C maps: the caller's rows, or the widened float32 copy when B / C are bf16
static bool make_bc_maps(const ssm_params_t* p, const Geo& g, const float* Bw, const float* Cw, CUtensorMap* tB,
                         CUtensorMap* tC) {
  if (g.bcbf16) {
    const uint64_t rs = kN * 4;
    return make_map(tB, Bw, false, kN, g.L, g.B, rs, (uint64_t)g.L * rs, kN, kChunk) &&
           make_map(tC, Cw, false, kN, g.L, g.B, rs, (uint64_t)g.L * rs, kN, kChunk);
  }
  const uint64_t rs = g.bs * 4;
  return make_map(tB, p->Bm, false, kN, g.L, g.B, rs, (uint64_t)g.L * rs, kN, kChunk) &&
         make_map(tC, p->Cm, false, kN, g.L, g.B, rs, (uint64_t)g.L * rs, kN, kChunk);
}

// ---------------------------------------------------------------- forward launch
static int fill_fwd_dir(const ssm_params_t* p, const Geo& g, FwdDir* d, cudaStream_t s, int box = kTileCh) {
  const uint64_t es = g.es;
  char* ws = static_cast<char*>(p->workspace);
  float* Bw = g.bcbf16 ? reinterpret_cast<float*>(ws + fwd_seg_bytes(g)) : nullptr;
  float* Cw = g.bcbf16 ? reinterpret_cast<float*>(ws + fwd_seg_bytes(g) + wide_bc_bytes(g) / 2) : nullptr;
  if (g.bcbf16) {
    const int st = launch_widen_bc(p, g, Bw, Cw, s);
    if (st) return st;
  }
  bool ok = make_map(&d->tm_u, p->u, g.bf16, g.Dm, g.L, g.B, g.Dm * es, (uint64_t)g.L * g.Dm * es, box, kChunk);
  ok = ok && make_map(&d->tm_delta, p->delta, g.bf16, g.Dm, g.L, g.B, g.Dm * es, (uint64_t)g.L * g.Dm * es,
                      box, kChunk);
  ok = ok && make_bc_maps(p, g, Bw, Cw, &d->tm_B, &d->tm_C);
  if (p->z)
    ok = ok && make_map(&d->tm_z, p->z, g.bf16, g.Dm, g.L, g.B, g.zs * es, (uint64_t)g.L * g.zs * es, box,
                        kChunk);
  else
    std::memset(&d->tm_z, 0, sizeof(d->tm_z));
  if (!ok) return SSM_ERR_LAUNCH;  // detail recorded by make_map
  d->A = p->A;
  d->D = p->D;
  d->bias = p->delta_bias;
  d->out = p->out;
  d->states = p->states;
  d->status = p->status;
  d->out_stride = g.os;
  d->L = g.L;
  d->Dm = g.Dm;
  d->flags = p->flags;
  d->gate_act = p->z ? p->gate_act : SSM_ACT_NONE;
  d->has_z = p->z != nullptr;
  const Seg sg = choose_segments(g, kFwdSeg);
  d->nseg = sg.nseg;
  d->seg_chunks = sg.seg_chunks;
  if (sg.nseg > 1) {
    char* ws = static_cast<char*>(p->workspace);
    const size_t rows = (size_t)g.B * sg.nseg * g.Dm;
    d->segI = reinterpret_cast<float*>(ws);
    ws += round256(rows * kN * 4);
    int* flags = reinterpret_cast<int*>(ws);
    d->seg_flag = flags + 4;  // after the ticket word
    // lookback flags (and the ticket) start at zero on every call
    SSM_CUDA_CHECK(cudaMemsetAsync(flags, 0, flag_bytes(g, sg.nseg, kTileCh), s), "cudaMemsetAsync(lookback flags)");
  }
  return SSM_OK;
}

// Shapes and flags the frame-specialised ("fast") kernel instances serve:
// softplus(dt), whole 16-step chunks, whole channel tiles.
static bool fast_shape(const Geo& g, int tile, int flags) {
  return (flags & SSM_DELTA_SOFTPLUS) && g.L % kChunk == 0 && g.Dm % tile == 0;
}

template <typename T, typename TBC>
static int launch_fwd_t(FwdLaunch& L, int ndir, const Geo& g, cudaStream_t s) {
  constexpr int kBytes = FwdSmem<T, TBC>::kBytes;
  const int nseg = L.dir[0].nseg;
  dim3 grid((g.Dm + kTileCh - 1) / kTileCh, g.B, 1);
  L.zdiv = nseg;
  grid.z = ndir * nseg;
  L.ntile = (int)grid.x;
  L.batch = g.B;
  L.chains = (int)grid.x * g.B * ndir;
  L.ticket = nseg > 1 ? L.dir[0].seg_flag - 4 : nullptr;
  L.spin_limit = kLookbackSpin;
  const bool wide = (long)grid.x * grid.y * grid.z <= (long)(kFMinBlocks / 2) * kSMs;
  const int fr = ndir == 1 && fast_shape(g, kTileCh, L.dir[0].flags) ? ((L.dir[0].flags & SSM_REVERSE) ? 2 : 1) : 0;
  auto pick = [&](auto fr_c) {
    constexpr int F = decltype(fr_c)::value;
    return nseg > 1 ? (wide ? ssm_fwd_kernel<T, TBC, true, true, F> : ssm_fwd_kernel<T, TBC, false, true, F>)
                    : (wide ? ssm_fwd_kernel<T, TBC, true, false, F> : ssm_fwd_kernel<T, TBC, false, false, F>);
  };
  auto kern = fr == 1 ? pick(std::integral_constant<int, 1>{})
                      : fr == 2 ? pick(std::integral_constant<int, 2>{}) : pick(std::integral_constant<int, 0>{});
  SSM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBytes),
                 "cudaFuncSetAttribute(ssm_fwd_kernel)");
  kern<<<grid, kFThreads, kBytes, s>>>(L);
  note_launches(1);
  SSM_CUDA_CHECK(cudaGetLastError(), "launch ssm_fwd_kernel");
  return SSM_OK;
}

// The one-lane-per-channel forward (scan_fwd_lane.cuh): single-direction,
// forward-frame launches of the fast shape without segments, with enough
// (batch row, channel) pairs to fill the GPU one lane each.
static bool lane_fwd(const Geo& g, int flags) {
#ifdef SSM_EXP_ENV
  if (const char* e = getenv("SSM_LANE"))
    if (atoi(e) == 0) return false;
#endif
  return g.ndir == 1 && !(flags & SSM_REVERSE) && fast_shape(g, kLTile, flags) &&
         (long)g.B * g.Dm >= kLaneMinChannels && choose_segments(g, kFwdSeg).nseg == 1;
}

template <typename T>
static int launch_fwd_lane_t(FwdLaunch& L, const Geo& g, cudaStream_t s) {
  constexpr int kBytes = LaneSmem<T>::kBytes;
  auto kern = ssm_fwd_lane_kernel<T, -1>;
  switch (L.dir[0].has_z ? L.dir[0].gate_act : -1) {
    case SSM_ACT_SILU: kern = ssm_fwd_lane_kernel<T, SSM_ACT_SILU>; break;
    case SSM_ACT_GELU: kern = ssm_fwd_lane_kernel<T, SSM_ACT_GELU>; break;
    case SSM_ACT_RELU: kern = ssm_fwd_lane_kernel<T, SSM_ACT_RELU>; break;
    case SSM_ACT_NONE: kern = ssm_fwd_lane_kernel<T, SSM_ACT_NONE>; break;
    default: break;
  }
  SSM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBytes),
                 "cudaFuncSetAttribute(ssm_fwd_lane_kernel)");
  kern<<<dim3(g.Dm / kLTile, g.B, 1), kLThreads, kBytes, s>>>(L);
  note_launches(1);
  SSM_CUDA_CHECK(cudaGetLastError(), "launch ssm_fwd_lane_kernel");
  return SSM_OK;
}

// B / C always reach the kernels as float32 (bf16 rows are widened first).
// A bidirectional call whose directions can both run frame-specialised
// instances runs them as two launches.
static int launch_fwd(FwdLaunch& L, int ndir, const Geo& g, cudaStream_t s) {
  if (ndir == 2 && fast_shape(g, kTileCh, L.dir[0].flags) && fast_shape(g, kTileCh, L.dir[1].flags)) {
    FwdLaunch L1 = L;
    L1.dir[0] = L.dir[1];
    const int st = launch_fwd(L, 1, g, s);
    return st ? st : launch_fwd(L1, 1, g, s);
  }
  if (g.bf16) return launch_fwd_t<__nv_bfloat16, float>(L, ndir, g, s);
  return launch_fwd_t<float, float>(L, ndir, g, s);
}

// ---------------------------------------------------------------- backward launch
struct BwdWs {
  float *dA_part, *dD_part, *db_part, *bc_part, *dB_acc, *dC_acc, *segI, *Bw, *Cw;
  int* flags;  // ticket word, then the lookback flags (null without segments)
  size_t flag_bytes;
  int64_t acc_stride;
};

static void carve_ws(const ssm_params_t* p, const Geo& g, char* ws, BwdWs* w, float* dbc_mc) {
  const Seg sg = choose_segments(g, kBwdSeg);
  const size_t rows = (size_t)g.B * sg.nseg * g.Dm;
  w->dA_part = reinterpret_cast<float*>(ws);
  ws += round256(rows * kN * 4);
  w->dD_part = reinterpret_cast<float*>(ws);
  ws += round256(rows * 4);
  w->db_part = reinterpret_cast<float*>(ws);
  ws += round256(rows * 4);
  w->segI = nullptr;
  w->flags = nullptr;
  w->flag_bytes = 0;
  if (sg.nseg > 1) {
    w->segI = reinterpret_cast<float*>(ws);
    ws += round256(rows * kN * 4);
    w->flags = reinterpret_cast<int*>(ws);
    w->flag_bytes = bwd_flag_bytes(g, sg.nseg);
    ws += w->flag_bytes;
  }
  w->bc_part = w->dB_acc = w->dC_acc = nullptr;
  w->acc_stride = kN;
  if (dbc_mc) {  // the partial sums go to the caller's multicast buffer (dense rows)
    w->dB_acc = dbc_mc;
    w->dC_acc = dbc_mc + (size_t)g.B * g.L * kN;
  } else {
    w->bc_part = reinterpret_cast<float*>(ws);
    ws += bc_part_bytes(g);
  }
  if (g.bcbf16) {
    w->Bw = reinterpret_cast<float*>(ws);
    w->Cw = reinterpret_cast<float*>(ws + wide_bc_bytes(g) / 2);
  } else {
    w->Bw = w->Cw = nullptr;
  }
}

static int fill_bwd_dir(const ssm_params_t* p, const Geo& g, const BwdWs& w, BwdDir* d, cudaStream_t s,
                        bool multicast) {
  const uint64_t es = g.es;
  if (g.bcbf16) {
    const int st = launch_widen_bc(p, g, w.Bw, w.Cw, s);
    if (st) return st;
  }
  bool ok = make_map(&d->tm_u, p->u, g.bf16, g.Dm, g.L, g.B, g.Dm * es, (uint64_t)g.L * g.Dm * es, kBTile, kChunk);
  ok = ok && make_map(&d->tm_delta, p->delta, g.bf16, g.Dm, g.L, g.B, g.Dm * es, (uint64_t)g.L * g.Dm * es,
                      kBTile, kChunk);
  ok = ok && make_bc_maps(p, g, w.Bw, w.Cw, &d->tm_B, &d->tm_C);
  ok = ok && make_map(&d->tm_dout, p->dout, g.bf16, g.Dm, g.L, g.B, g.os * es, (uint64_t)g.L * g.os * es, kBTile,
                      kChunk);
  if (p->z)
    ok = ok && make_map(&d->tm_z, p->z, g.bf16, g.Dm, g.L, g.B, g.zs * es, (uint64_t)g.L * g.zs * es, kBTile,
                        kChunk);
  else
    std::memset(&d->tm_z, 0, sizeof(d->tm_z));
  if (!ok) return SSM_ERR_LAUNCH;  // detail recorded by make_map
  d->states = p->states;
  d->A = p->A;
  d->D = p->D;
  d->bias = p->delta_bias;
  d->du = p->du;
  d->ddelta = p->ddelta;
  d->dz = p->dz;
  d->bc_part = w.bc_part;
  d->dB_acc = w.dB_acc;
  d->dC_acc = w.dC_acc;
  d->bc_mode = multicast ? kBcMulticast : kBcLocal;
  d->dA_part = w.dA_part;
  d->dD_part = w.dD_part;
  d->db_part = w.db_part;
  d->status = p->status;
  d->z_stride = g.zs;
  d->acc_stride = w.acc_stride;
  d->L = g.L;
  d->Dm = g.Dm;
  d->flags = p->flags;
  d->gate_act = p->z ? p->gate_act : SSM_ACT_NONE;
  d->has_z = p->z != nullptr;
  const Seg sg = choose_segments(g, kBwdSeg);
  d->nseg = sg.nseg;
  d->seg_chunks = sg.seg_chunks;
  d->segI = w.segI;
  d->seg_flag = w.flags ? w.flags + 4 : nullptr;
  return SSM_OK;
}

// Test hook of the lookback failure path: the launch leaves out the CTAs of
// the last segment (their tickets are skipped), so the segment before it
// waits for a flag that is never set and gives up after spin_limit polls.
struct BwdHook {
  uint32_t spin_limit;
  bool drop_last_segment;
};

template <typename T, typename TBC, int G>
static int launch_bwd_t(BwdLaunch& L, int ndir, const Geo& g, cudaStream_t s, const BwdHook* hook) {
  int bytes = 0;
  for (int d = 0; d < ndir; ++d) {
    const BwdDir& a = L.dir[d];
    const bool mirror = a.D && (a.flags & SSM_REVERSE) && !(a.flags & SSM_ALIGNED_SKIP);
    const BwdLayout lay(sizeof(T), sizeof(TBC), a.has_z != 0, mirror);
    bytes = lay.bytes > bytes ? lay.bytes : bytes;
  }
  const int nseg = L.dir[0].nseg;
  dim3 grid((g.Dm + kBTile - 1) / kBTile, g.B, 1);
  const BwdDir& d0 = L.dir[0];
  const int fr = ndir == 1 && fast_shape(g, kBTile, d0.flags) ? ((d0.flags & SSM_REVERSE) ? 2 : 1) : 0;
  const bool mc = d0.bc_mode == kBcMulticast;
  // The flavoured instances exist with and without the segment code; the
  // generic one always carries it.  The multicast form (d_inner sharding) has
  // no reverse-frame instance.
  const bool seg = nseg > 1;
  auto kern = ssm_bwd_kernel<T, TBC, G, false, 0, true>;
  if (mc) {
    kern = fr == 1 ? (seg ? ssm_bwd_kernel<T, TBC, G, true, 1, true> : ssm_bwd_kernel<T, TBC, G, true, 1, false>)
                   : ssm_bwd_kernel<T, TBC, G, true, 0, true>;
  } else if (fr == 1) {
    kern = seg ? ssm_bwd_kernel<T, TBC, G, false, 1, true> : ssm_bwd_kernel<T, TBC, G, false, 1, false>;
  } else if (fr == 2) {
    kern = seg ? ssm_bwd_kernel<T, TBC, G, false, 2, true> : ssm_bwd_kernel<T, TBC, G, false, 2, false>;
  }
  SSM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                 "cudaFuncSetAttribute(ssm_bwd_kernel)");
  L.zdiv = nseg;
  grid.z = ndir * nseg;
  L.ntile = (int)grid.x;
  L.batch = g.B;
  L.chains = (int)grid.x * g.B * ndir;
  if (hook) {
    L.spin_limit = hook->spin_limit;
    if (hook->drop_last_segment) {
      grid.z = ndir * (nseg - 1);
      L.ticket_base = L.chains;
    }
  }
  kern<<<grid, kBThreads, bytes, s>>>(L);
  note_launches(1);
  SSM_CUDA_CHECK(cudaGetLastError(), "launch ssm_bwd_kernel");
  return SSM_OK;
}

template <typename T, typename TBC>
static int launch_bwd_g(BwdLaunch& L, int ndir, const Geo& g, cudaStream_t s, const BwdHook* hook) {
  if (!L.dir[0].has_z) return launch_bwd_t<T, TBC, -1>(L, ndir, g, s, hook);
  switch (L.dir[0].gate_act) {
    case SSM_ACT_SILU: return launch_bwd_t<T, TBC, SSM_ACT_SILU>(L, ndir, g, s, hook);
    case SSM_ACT_GELU: return launch_bwd_t<T, TBC, SSM_ACT_GELU>(L, ndir, g, s, hook);
    case SSM_ACT_RELU: return launch_bwd_t<T, TBC, SSM_ACT_RELU>(L, ndir, g, s, hook);
    default: return launch_bwd_t<T, TBC, SSM_ACT_NONE>(L, ndir, g, s, hook);
  }
}

static int launch_bwd(BwdLaunch& L, int ndir, const Geo& g, cudaStream_t s, const BwdHook* hook) {
  // One launch per direction when the gates differ, or when both directions
  // can run a frame-specialised instance (frame, softplus and masks
  // compile-time), which beats sharing one generic launch.
  if (ndir == 2 && (L.dir[0].gate_act != L.dir[1].gate_act || L.dir[0].has_z != L.dir[1].has_z ||
                    (fast_shape(g, kBTile, L.dir[0].flags) && fast_shape(g, kBTile, L.dir[1].flags) &&
                     L.dir[0].bc_mode != kBcMulticast))) {
    BwdLaunch L1 = L;
    L1.dir[0] = L.dir[1];
    if (L.ticket) {  // the second launch takes its tickets from the second direction's word
      L1.ticket = L.dir[1].seg_flag - 4;
    }
    const int st = launch_bwd(L, 1, g, s, hook);
    return st ? st : launch_bwd(L1, 1, g, s, hook);
  }
  if (g.bf16) return launch_bwd_g<__nv_bfloat16, float>(L, ndir, g, s, hook);  // B / C widened to float32
  return launch_bwd_g<float, float>(L, ndir, g, s, hook);
}

static int launch_finalize(const ssm_params_t* p, const Geo& g, const BwdWs& w, cudaStream_t s, bool reduced) {
  FinalizeDir f;
  f.dA_part = w.dA_part;
  f.dD_part = w.dD_part;
  f.db_part = w.db_part;
  f.dA = p->dA;
  f.dD = p->D ? p->dD : nullptr;
  f.dbias = p->delta_bias ? p->ddelta_bias : nullptr;
  f.bc_part = reduced ? nullptr : w.bc_part;
  f.dB = p->dB;
  f.dC = p->dC;
  f.bc_stride = g.bs;
  f.prows = g.B * choose_segments(g, kBwdSeg).nseg;
  f.ntile = (g.Dm + kBTile - 1) / kBTile;
  f.batch = g.B;
  f.L = g.L;
  f.Dm = g.Dm;
  const int threads = 256;
  int64_t n = (int64_t)g.Dm * kN;
  unsigned blocks = (unsigned)((n + threads - 1) / threads);
  if (f.bc_part) {  // enough threads for the dB / dC rows (grid-stride beyond 8 CTAs per SM)
    const int64_t nbc = ((int64_t)g.B * g.L * 8 + threads - 1) / threads;
    const int64_t cap = 8L * kSMs;
    const unsigned want = (unsigned)(nbc < cap ? nbc : cap);
    blocks = blocks < want ? want : blocks;
  }
  if (blocks == 0) return SSM_OK;
  if (g.bcbf16)
    finalize_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(f);
  else
    finalize_kernel<float><<<blocks, threads, 0, s>>>(f);
  note_launches(1);
  SSM_CUDA_CHECK(cudaGetLastError(), "launch finalize_kernel");
  return SSM_OK;
}

static bool same_geo(const Geo& a, const Geo& b) {
  return a.B == b.B && a.L == b.L && a.Dm == b.Dm && a.bf16 == b.bf16 && a.bcbf16 == b.bcbf16;
}

}  // namespace ssm

using namespace ssm;

extern "C" {

size_t ssm_states_elems(const ssm_params_t* p) {
  if (!p || p->batch <= 0 || p->seqlen <= 0 || p->dim <= 0) return 0;
  return (size_t)p->batch * ((p->seqlen + kCk - 1) / kCk) * p->dim * kN;
}

size_t ssm_workspace_bytes(const ssm_params_t* p) {
  Geo g;
  if (check_common(p, &g) != SSM_OK) return 0;
  return ws_bytes(g);
}

size_t ssm_bwd_workspace_bytes(const ssm_params_t* p, int multicast) {
  Geo g;
  if (check_common(p, &g) != SSM_OK) return 0;
  return bwd_ws_bytes(g, multicast != 0);
}

size_t ssm_fwd_workspace_bytes(const ssm_params_t* p) {
  Geo g;
  if (check_common(p, &g) != SSM_OK) return 0;
  if ((int64_t)g.B * g.L * g.Dm == 0) return 0;
  return fwd_ws_bytes(g);
}

int ssm_fwd(const ssm_params_t* p, ssm_stream_t stream) { return ssm_fwd_bidir(p, nullptr, stream); }

int ssm_fwd_bidir(const ssm_params_t* fwd, const ssm_params_t* rev, ssm_stream_t stream) {
  Geo g, g2;
  int st = check_fwd(fwd, &g);
  if (st) return st;
  if (rev) {
    st = check_fwd(rev, &g2);
    if (st) return st;
    if (!same_geo(g, g2)) return SSM_ERR_SHAPE;
    g.ndir = 2;
  }
  if ((int64_t)g.B * g.L * g.Dm == 0) return SSM_OK;
  st = bind_device(fwd->u);
  if (st) return st;
  const size_t need = fwd_ws_bytes(g);
  for (const ssm_params_t* q : {fwd, rev}) {
    if (!q) continue;
    if (need && (!q->workspace || q->workspace_bytes < need)) return SSM_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(q->workspace) & 255u) return SSM_ERR_ALIGN;
  }
  FwdLaunch args;
  std::memset(&args, 0, sizeof(args));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (lane_fwd(g, fwd->flags)) {
    st = fill_fwd_dir(fwd, g, &args.dir[0], s, kLTile);
    if (st) return st;
    return g.bf16 ? launch_fwd_lane_t<__nv_bfloat16>(args, g, s) : launch_fwd_lane_t<float>(args, g, s);
  }
  st = fill_fwd_dir(fwd, g, &args.dir[0], s);
  if (!st && rev) st = fill_fwd_dir(rev, g, &args.dir[1], s);
  if (st) return st;
  return launch_fwd(args, rev ? 2 : 1, g, s);
}

namespace ssm {
static int bwd_impl(const ssm_params_t* fwd, const ssm_params_t* rev, float* dbc_mc, ssm_stream_t stream,
                    const BwdHook* hook = nullptr) {
  Geo g, g2;
  int st = check_bwd(fwd, &g);
  if (st) return st;
  if (rev) {
    st = check_bwd(rev, &g2);
    if (st) return st;
    if (!same_geo(g, g2)) return SSM_ERR_SHAPE;
    g.ndir = 2;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  st = bind_device((int64_t)g.B * g.L * g.Dm ? fwd->u : (const void*)fwd->dA);
  if (st) return st;
  const size_t need = bwd_ws_bytes(g, dbc_mc != nullptr) * (rev ? 2 : 1);
  if (need && (!fwd->workspace || fwd->workspace_bytes < need)) return SSM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(fwd->workspace) & 255u) return SSM_ERR_ALIGN;
  BwdWs w[2];
  carve_ws(fwd, g, static_cast<char*>(fwd->workspace), &w[0], dbc_mc);
  if (rev) carve_ws(rev, g, static_cast<char*>(fwd->workspace) + bwd_ws_bytes(g, dbc_mc != nullptr), &w[1], dbc_mc);
  const int ndir = rev ? 2 : 1;
  const ssm_params_t* ps[2] = {fwd, rev};
  if ((int64_t)g.B * g.L * g.Dm == 0) {
    // nothing to scan: parameter gradients are zero
    for (int d = 0; d < ndir; ++d) {
      if (g.Dm == 0) continue;
      SSM_CUDA_CHECK(cudaMemsetAsync(ps[d]->dA, 0, (size_t)g.Dm * kN * 4, s), "cudaMemsetAsync(dA)");
      if (ps[d]->D) SSM_CUDA_CHECK(cudaMemsetAsync(ps[d]->dD, 0, (size_t)g.Dm * 4, s), "cudaMemsetAsync(dD)");
      if (ps[d]->delta_bias)
        SSM_CUDA_CHECK(cudaMemsetAsync(ps[d]->ddelta_bias, 0, (size_t)g.Dm * 4, s), "cudaMemsetAsync(dbias)");
    }
    return SSM_OK;
  }
  BwdLaunch args;
  std::memset(&args, 0, sizeof(args));
  for (int d = 0; d < ndir; ++d) {
    st = fill_bwd_dir(ps[d], g, w[d], &args.dir[d], s, dbc_mc != nullptr);
    if (st) return st;
    if (w[d].flags)  // lookback flags (and the ticket) start at zero on every call
      SSM_CUDA_CHECK(cudaMemsetAsync(w[d].flags, 0, w[d].flag_bytes, s), "cudaMemsetAsync(lookback flags)");
  }
  args.ticket = w[0].flags;
  args.spin_limit = kLookbackSpin;
  if (hook && (!w[0].flags || hook->spin_limit == 0)) return SSM_ERR_SHAPE;  // the self-test needs segments
  st = launch_bwd(args, ndir, g, s, hook);
  if (st) return st;
  for (int d = 0; d < ndir; ++d) {
    st = launch_finalize(ps[d], g, w[d], s, dbc_mc != nullptr);
    if (st) return st;
  }
  return SSM_OK;
}
}  // namespace ssm

int ssm_bwd(const ssm_params_t* p, ssm_stream_t stream) { return bwd_impl(p, nullptr, nullptr, stream); }

int ssm_bwd_bidir(const ssm_params_t* fwd, const ssm_params_t* rev, ssm_stream_t stream) {
  return bwd_impl(fwd, rev, nullptr, stream);
}

int ssm_bwd_bc_multicast(const ssm_params_t* p, float* dbc_mc, ssm_stream_t stream) {
  if (!p || !dbc_mc) return SSM_ERR_NULL;
  if (!aligned16(dbc_mc)) return SSM_ERR_ALIGN;
  // dB / dC go to the multicast buffer: stand-ins keep ssm_bwd's pointer
  // checks meaningful for everything else
  ssm_params_t q = *p;
  q.dB = dbc_mc;
  q.dC = dbc_mc;
  return bwd_impl(&q, nullptr, dbc_mc, stream);
}

int ssm_selftest_lookback_timeout(const ssm_params_t* p, uint32_t spin_limit, ssm_stream_t stream) {
  if (!p || !p->status) return SSM_ERR_NULL;
  if (spin_limit == 0 || spin_limit > kLookbackSpin) return SSM_ERR_SHAPE;
  const BwdHook hook{spin_limit, true};
  return bwd_impl(p, nullptr, nullptr, stream, &hook);
}

const char* ssm_strerror(int status) {
  switch (status) {
    case SSM_OK: return "ok";
    case SSM_ERR_SHAPE: return "unsupported or inconsistent shape (dstate must be 16; batch <= 65535)";
    case SSM_ERR_DTYPE: return "unsupported dtype code";
    case SSM_ERR_LAUNCH: return "CUDA launch or driver error";
    case SSM_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case SSM_ERR_NULL: return "a required pointer is NULL";
    case SSM_ERR_ALIGN: return "pointer or row stride not 16-byte aligned (dim*elem_size must be a multiple of 16)";
    case SSM_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    default: return "unknown status";
  }
}

unsigned long long ssm_launch_count(void) { return ssm::g_launches.load(std::memory_order_relaxed); }

const char* ssm_version(void) { return "selectssm_b200 0.1.0 (sm_100a)"; }

const char* ssm_last_error(void) { return g_last_error; }

}  // extern "C"
