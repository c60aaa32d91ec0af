// Causal depthwise conv1d + activation preamble of SelectiveSSM
// (src/selectssm/selectssm.py:167-187) and its gradient, reading the flipped
// (reverse) or flipped-and-complemented sequence in place instead of
// materialising jnp.flip copies.
//
// Thread = one channel x a segment of kSeg consecutive steps; a warp covers 32
// consecutive channels, so every load and store is a coalesced 128-byte row
// (the complement flip maps a warp's channels onto a reversed but still
// contiguous row).  The K-tap window lives in registers.
#include "common.cuh"
#include "../../include/selectssm_b200.h"

namespace ssm {

int launch_error(const char* where, cudaError_t e);  // scan.cu
int bind_device(const void* ptr);                      // scan.cu

constexpr int kConvMaxK = 8;
constexpr int kSeg = 64;      // steps per thread
constexpr int kConvCh = 32;   // channels per block row
constexpr int kConvSegs = 4;  // segments per block

struct ConvArgs {
  const void* x;
  const float* w;
  void* u;
  const void* du;
  void* dx;
  float* dw_part;  // (B, nsegblk, K, D)
  int64_t xs;      // row stride of x / dx
  int L, Dm, K, act, rev, comp, nsegblk;
};

template <typename T>
__device__ __forceinline__ float load_xt(const ConvArgs& a, int b, int t, int c) {
  // x~[t, c] with the flip of selectssm.py:168 folded into the index
  if (t < 0 || t >= a.L) return 0.f;
  const int l = a.rev ? a.L - 1 - t : t;
  const int cc = a.comp ? a.Dm - 1 - c : c;
  return Cvt<T>::to_f(reinterpret_cast<const T*>(a.x)[((int64_t)b * a.L + l) * a.xs + cc]);
}

template <typename T>
__global__ void __launch_bounds__(kConvCh* kConvSegs) conv_fwd_kernel(const ConvArgs a) {
  const int c = blockIdx.x * kConvCh + threadIdx.x;
  const int seg = blockIdx.y * kConvSegs + threadIdx.y;
  const int b = blockIdx.z;
  if (c >= a.Dm) return;
  const int t0 = seg * kSeg;
  if (t0 >= a.L) return;
  float w[kConvMaxK], win[kConvMaxK];
#pragma unroll
  for (int k = 0; k < kConvMaxK; ++k) {
    w[k] = k < a.K ? a.w[(int64_t)k * a.Dm + c] : 0.f;
    win[k] = 0.f;
  }
  // window: win[k] holds x~[t - (K-1) + k]; prime with the K-1 steps before t0
  for (int k = 0; k < a.K - 1; ++k) win[k + 1] = load_xt<T>(a, b, t0 - (a.K - 1) + k, c);
  T* u = reinterpret_cast<T*>(a.u);
  const int t1 = min(t0 + kSeg, a.L);
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int k = 0; k < kConvMaxK - 1; ++k) win[k] = win[k + 1];
    // newest sample goes to slot K-1
    const float xn = load_xt<T>(a, b, t, c);
    float pre = 0.f;
#pragma unroll
    for (int k = 0; k < kConvMaxK; ++k) {
      const float xv = (k == a.K - 1) ? xn : win[k];
      if (k < a.K) pre = fmaf(w[k], xv, pre);
    }
#pragma unroll
    for (int k = 0; k < kConvMaxK; ++k)
      if (k == a.K - 1) win[k] = xn;
    u[((int64_t)b * a.L + t) * a.Dm + c] = Cvt<T>::from_f(act_f(pre, a.act));
  }
}

// Backward: dpre[t] = du[t] act'(pre[t]); dx~[t] = sum_k w[k] dpre[t + K-1-k];
// dw[k] = sum_t dpre[t] x~[t + k - (K-1)].  dx is written back in x's frame.
template <typename T>
__global__ void __launch_bounds__(kConvCh* kConvSegs) conv_bwd_kernel(const ConvArgs a) {
  const int c = blockIdx.x * kConvCh + threadIdx.x;
  const int seg = blockIdx.y * kConvSegs + threadIdx.y;
  const int b = blockIdx.z;
  const int t0 = seg * kSeg;
  float dw[kConvMaxK];
#pragma unroll
  for (int k = 0; k < kConvMaxK; ++k) dw[k] = 0.f;
  if (c < a.Dm && t0 < a.L) {
    float w[kConvMaxK], xw[2 * kConvMaxK], dp[kConvMaxK];
#pragma unroll
    for (int k = 0; k < kConvMaxK; ++k) {
      w[k] = k < a.K ? a.w[(int64_t)k * a.Dm + c] : 0.f;
      dp[k] = 0.f;
    }
    // xw[k] = x~[tau - (K-1) + k], k in [0, K), maintained for tau
#pragma unroll
    for (int k = 0; k < 2 * kConvMaxK; ++k) xw[k] = 0.f;
    for (int k = 0; k < a.K - 1; ++k) xw[k + 1] = load_xt<T>(a, b, t0 - (a.K - 1) + k, c);
    const T* du = reinterpret_cast<const T*>(a.du);
    T* dx = reinterpret_cast<T*>(a.dx);
    const int tend = min(t0 + kSeg, a.L);
    // tau runs K-1 steps past the segment so every dx~[t] of the segment is complete
    for (int tau = t0; tau < tend + a.K - 1; ++tau) {
#pragma unroll
      for (int k = 0; k < kConvMaxK - 1; ++k) xw[k] = xw[k + 1];
      const float xn = load_xt<T>(a, b, tau, c);
#pragma unroll
      for (int k = 0; k < kConvMaxK; ++k)
        if (k == a.K - 1) xw[k] = xn;
      float dpre = 0.f;
      if (tau < a.L) {
        float pre = 0.f;
#pragma unroll
        for (int k = 0; k < kConvMaxK; ++k)
          if (k < a.K) pre = fmaf(w[k], xw[k], pre);
        dpre = Cvt<T>::to_f(du[((int64_t)b * a.L + tau) * a.Dm + c]) * act_grad_f(pre, a.act);
        if (tau < tend) {
#pragma unroll
          for (int k = 0; k < kConvMaxK; ++k)
            if (k < a.K) dw[k] = fmaf(dpre, xw[k], dw[k]);
        }
      }
      // dp[k] holds dpre[tau - k]
#pragma unroll
      for (int k = kConvMaxK - 1; k > 0; --k) dp[k] = dp[k - 1];
      dp[0] = dpre;
      const int t = tau - (a.K - 1);  // dx~[t] = sum_k w[k] dpre[t + K-1-k] = sum_k w[k] dp[k]
      if (t >= t0) {
        float g = 0.f;
#pragma unroll
        for (int k = 0; k < kConvMaxK; ++k)
          if (k < a.K) g = fmaf(w[k], dp[k], g);
        const int l = a.rev ? a.L - 1 - t : t;
        const int cc = a.comp ? a.Dm - 1 - c : c;
        dx[((int64_t)b * a.L + l) * a.xs + cc] = Cvt<T>::from_f(g);
      }
    }
  }
  // dw partial per (batch row, segment block): reduce the block's segments in smem
  __shared__ float sdw[kConvSegs][kConvMaxK][kConvCh];
#pragma unroll
  for (int k = 0; k < kConvMaxK; ++k) sdw[threadIdx.y][k][threadIdx.x] = dw[k];
  __syncthreads();
  if (threadIdx.y == 0 && c < a.Dm) {
    for (int k = 0; k < a.K; ++k) {
      float s = 0.f;
      for (int q = 0; q < kConvSegs; ++q) s += sdw[q][k][threadIdx.x];
      a.dw_part[(((int64_t)b * a.nsegblk + blockIdx.y) * a.K + k) * a.Dm + c] = s;
    }
  }
}

__global__ void conv_dw_reduce_kernel(const float* part, float* dw, int rows, int K, int Dm) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over K*Dm
  if (i >= K * Dm) return;
  float s = 0.f;
  for (int r = 0; r < rows; ++r) s += part[(int64_t)r * K * Dm + i];
  dw[i] = s;
}

static int check_conv(const ssm_conv_params_t* p) {
  if (!p) return SSM_ERR_NULL;
  if (p->batch < 0 || p->seqlen < 0 || p->dim < 0 || p->width < 1 || p->width > kConvMaxK) return SSM_ERR_SHAPE;
  if (p->batch > 65535) return SSM_ERR_SHAPE;
  if (p->dtype != SSM_F32 && p->dtype != SSM_BF16) return SSM_ERR_DTYPE;
  if (p->act < SSM_ACT_NONE || p->act > SSM_ACT_RELU) return SSM_ERR_SHAPE;
  if (p->x_stride && p->x_stride < p->dim) return SSM_ERR_SHAPE;
  return SSM_OK;
}

static ConvArgs conv_args(const ssm_conv_params_t* p) {
  ConvArgs a;
  a.x = p->x;
  a.w = p->w;
  a.u = p->u;
  a.du = p->du;
  a.dx = p->dx;
  a.dw_part = static_cast<float*>(p->workspace);
  a.xs = p->x_stride ? p->x_stride : p->dim;
  a.L = p->seqlen;
  a.Dm = p->dim;
  a.K = p->width;
  a.act = p->act;
  a.rev = (p->flags & SSM_REVERSE) != 0;
  a.comp = a.rev && (p->flags & SSM_COMPLEMENT) != 0;
  a.nsegblk = (p->seqlen + kSeg * kConvSegs - 1) / (kSeg * kConvSegs);
  return a;
}

}  // namespace ssm

using namespace ssm;

extern "C" {

size_t ssm_conv1d_workspace_bytes(const ssm_conv_params_t* p) {
  if (check_conv(p) != SSM_OK) return 0;
  const size_t nsegblk = (p->seqlen + kSeg * kConvSegs - 1) / (kSeg * kConvSegs);
  return (size_t)p->batch * nsegblk * p->width * p->dim * sizeof(float);
}

int ssm_conv1d_act_fwd(const ssm_conv_params_t* p, ssm_stream_t stream) {
  int st = check_conv(p);
  if (st) return st;
  if ((int64_t)p->batch * p->seqlen * p->dim == 0) return SSM_OK;
  if (!p->x || !p->w || !p->u) return SSM_ERR_NULL;
  st = bind_device(p->x);
  if (st) return st;
  ConvArgs a = conv_args(p);
  dim3 block(kConvCh, kConvSegs);
  dim3 grid((a.Dm + kConvCh - 1) / kConvCh, a.nsegblk, p->batch);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->dtype == SSM_BF16)
    conv_fwd_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(a);
  else
    conv_fwd_kernel<float><<<grid, block, 0, s>>>(a);
  note_launches(1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SSM_OK : launch_error("launch conv_fwd_kernel", e);
}

int ssm_conv1d_act_bwd(const ssm_conv_params_t* p, ssm_stream_t stream) {
  int st = check_conv(p);
  if (st) return st;
  if (!p->dw) return SSM_ERR_NULL;
  st = bind_device(p->dw);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((int64_t)p->batch * p->seqlen * p->dim == 0) {
    if (p->dim) {
      const cudaError_t e = cudaMemsetAsync(p->dw, 0, (size_t)p->width * p->dim * 4, s);
      if (e != cudaSuccess) return launch_error("cudaMemsetAsync(dw)", e);
    }
    return SSM_OK;
  }
  if (!p->x || !p->w || !p->du || !p->dx) return SSM_ERR_NULL;
  if (!p->workspace || p->workspace_bytes < ssm_conv1d_workspace_bytes(p)) return SSM_ERR_WORKSPACE;
  ConvArgs a = conv_args(p);
  dim3 block(kConvCh, kConvSegs);
  dim3 grid((a.Dm + kConvCh - 1) / kConvCh, a.nsegblk, p->batch);
  if (p->dtype == SSM_BF16)
    conv_bwd_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(a);
  else
    conv_bwd_kernel<float><<<grid, block, 0, s>>>(a);
  const int n = a.K * a.Dm;
  conv_dw_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(a.dw_part, p->dw, p->batch * a.nsegblk, a.K, a.Dm);
  note_launches(2);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SSM_OK : launch_error("launch conv_bwd_kernel", e);
}

}  // extern "C"
