// Device helpers shared by the selective-scan kernels (sm_100a).
//
// Everything here is hand-written PTX for data movement (mbarrier, TMA tensor
// loads) and for the hardware special-function instructions (ex2/lg2/rcp).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ssm {

// Adds n to the library's count of kernels launched (ssm_launch_count).
void note_launches(unsigned n);

constexpr int kChunk = 16;        // steps per TMA stage
constexpr int kCk = 8;            // forward checkpoint spacing (backward register block)
constexpr int kN = 16;            // state size supported by this build
#ifndef SSM_FWD_TILE
#define SSM_FWD_TILE 32
#endif
constexpr int kTileCh = SSM_FWD_TILE;  // channels per forward CTA (the TMA box width)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// Upper bound on polls of an mbarrier before a kernel gives up (each poll of
// try_wait suspends for a hardware-defined time, so this is seconds, not a
// tight loop).
constexpr uint32_t kSpinLimit = 1u << 24;

// error codes written to the optional status word
constexpr int kStatusTimeout = 4;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false if the barrier did not complete within `limit`
// polls (kSpinLimit, well above any legitimate wait, unless given).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit = kSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ---------------------------------------------------------------- TMA
// 3-D tiled tensor load (no multicast): box lands at `dst`, completion counted
// on `bar` in bytes.  Coordinates are (channel, step, batch); the channel
// coordinate times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tensor memory
// TMEM (256 KB per SM) holds per-thread scratch the register file cannot: a
// warp reads and writes its own 32-lane quarter (warp_id % 4) of the 128 lanes.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 8 consecutive columns of this thread's lane
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
// 16 consecutive columns of this thread's lane (completes at tmem_wait_ld)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- cross-GPU reduction
// Adds v to the 4 floats at an NVLink multicast address: the NVSwitch applies
// the add to the copy on every GPU bound to the multicast object.
__device__ __forceinline__ void multimem_red_add4(float* mc, float4 v) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softplus(x) = log(1 + e^x).  For x < -3 the Taylor series of log1p(e)
// (e = e^x < 0.05; six terms, relative truncation below 3e-9) avoids the
// cancellation of log(1 + small); for x > 20 softplus(x) == x in fp32.  Both
// forms are evaluated and selected, so a warp never branches on the data.
__device__ __forceinline__ float softplus_f(float x) {
  const float e = ex2(fminf(x, 20.f) * kLog2e);
  const float p = 0.2f - e * (1.f / 6.f);
  const float series = e * (1.f - e * (0.5f - e * (1.f / 3.f - e * (0.25f - e * p))));
  const float r = x < -3.f ? series : lg2(1.f + e) * kLn2;
  return x > 20.f ? x : r;
}
// softplus(x) and its derivative sigmoid(x) = e / (1 + e), e = e^x, from one
// exponential (same forms and ranges as softplus_f).
__device__ __forceinline__ float softplus_sig(float x, float& sig) {
  const float e = ex2(fminf(x, 20.f) * kLog2e);
  sig = x > 20.f ? 1.f : e * rcp(1.f + e);
  const float p = 0.2f - e * (1.f / 6.f);
  const float series = e * (1.f - e * (0.5f - e * (1.f / 3.f - e * (0.25f - e * p))));
  const float r = x < -3.f ? series : lg2(1.f + e) * kLn2;
  return x > 20.f ? x : r;
}
// logistic sigmoid
__device__ __forceinline__ float sigmoid_f(float x) { return rcp(1.f + ex2(-x * kLog2e)); }

// tanh from the exponential: tanh(x) = 1 - 2 / (1 + e^{2x}) (absolute error
// ~1e-7, which is what the gelu gate needs).
__device__ __forceinline__ float tanh_f(float x) {
  x = fminf(fmaxf(x, -15.f), 15.f);
  return 1.f - 2.f * rcp(1.f + ex2(2.f * kLog2e * x));
}

constexpr float kGeluC = 0.7978845608028654f;  // sqrt(2/pi)

// activation and its derivative; act is an ssm_act code
__device__ __forceinline__ float act_f(float x, int act) {
  switch (act) {
    case 1: return x * sigmoid_f(x);
    case 2: return 0.5f * x * (1.f + tanh_f(kGeluC * (x + 0.044715f * x * x * x)));
    case 3: return fmaxf(x, 0.f);
    default: return x;
  }
}
__device__ __forceinline__ float act_grad_f(float x, int act) {
  switch (act) {
    case 1: {
      const float s = sigmoid_f(x);
      return s * (1.f + x * (1.f - s));
    }
    case 2: {
      const float t = tanh_f(kGeluC * (x + 0.044715f * x * x * x));
      const float di = kGeluC * (1.f + 3.f * 0.044715f * x * x);
      return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * di;
    }
    case 3: return x > 0.f ? 1.f : 0.f;
    default: return 1.f;
  }
}

// act(x) and act'(x) together, sharing the exponential / tanh
__device__ __forceinline__ void act_and_grad(float x, int act, float& a, float& g) {
  switch (act) {
    case 1: {
      const float s = sigmoid_f(x);
      a = x * s;
      g = s * (1.f + x * (1.f - s));
      return;
    }
    case 2: {
      const float t = tanh_f(kGeluC * (x + 0.044715f * x * x * x));
      const float di = kGeluC * (1.f + 3.f * 0.044715f * x * x);
      a = 0.5f * x * (1.f + t);
      g = 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * di;
      return;
    }
    case 3:
      a = fmaxf(x, 0.f);
      g = x > 0.f ? 1.f : 0.f;
      return;
    default:
      a = x;
      g = 1.f;
  }
}

// ---------------------------------------------------------------- packed fp32 (sm_100 f32x2)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 dup2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x for a pair of values on the FMA / integer pipes instead of the MUFU
// unit (which issues a quarter as fast), so kernels that need many
// exponentials can split them over both.  Method: clamp x to [-126, 126];
// round to j = rint(x) by adding and subtracting 1.5 * 2^23 (j then sits in the
// low mantissa bits of the sum); f = x - j lies in [-1/2, 1/2]; 2^f is a
// degree-5 polynomial whose coefficients were fitted for the smallest maximum
// relative error on that interval (iteratively reweighted least squares,
// Lawson's algorithm); the result is 2^f with j added to its exponent field.
// Maximum relative error 2.4e-7 (checked on a dense grid by the CPU tests).
constexpr float kExp2P0 = 1.0000001192092896f, kExp2P1 = 0.6931469440460205f, kExp2P2 = 0.24022120237350464f,
                kExp2P3 = 0.05550713092088699f, kExp2P4 = 0.009675541892647743f, kExp2P5 = 0.001327647129073739f;
constexpr float kRoundMagic = 12582912.f;  // 1.5 * 2^23
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fminf(fmaxf(x.x, -126.f), 126.f);
  x.y = fminf(fmaxf(x.y, -126.f), 126.f);
  const float2 t = fadd2(x, dup2(kRoundMagic));
  const float2 f = fsub2(x, fsub2(t, dup2(kRoundMagic)));
  float2 p = ffma2(dup2(kExp2P5), f, dup2(kExp2P4));
  p = ffma2(p, f, dup2(kExp2P3));
  p = ffma2(p, f, dup2(kExp2P2));
  p = ffma2(p, f, dup2(kExp2P1));
  p = ffma2(p, f, dup2(kExp2P0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// ---------------------------------------------------------------- dtype helpers
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <> struct Cvt<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <typename T> __device__ __forceinline__ float ld_f(const T* p) { return Cvt<T>::to_f(*p); }

// four consecutive values (16-byte aligned for float, 8-byte for bf16)
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 r = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
  __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
  const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status) atomicExch(status, code);
}

}  // namespace ssm
