// RMSNorm around BidirectionalMamba (src/selectssm/selectssm.py:306-313 with
// norm_type "rms", flax.linen.RMSNorm: y = x * rsqrt(mean(x^2) + eps) * scale)
// and the residual base of the block's output (selectssm.py:345-352:
// out = skip + out_proj(h), out_proj(h) = h W + b).
//
// The forward reads each row of x once and writes both the normalised row and
// base = x + b, so the out_proj GEMM can take the residual and its bias as the
// accumulator operand of one cuBLAS call (out = base + h W).  The backward
// computes dx and per-block partials of dscale, summed in a fixed order by a
// second kernel (deterministic).
//
// Layout: rows of `dim` contiguous elements (fp32 or bf16), fp32 scale and
// per-row rstd.  One warp per row; each lane holds dim/32 elements in
// registers (dim <= 32 * kMaxPerLane), so a row is read once per pass.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "../../include/selectssm_b200.h"

namespace ssm {

int launch_error(const char* where, cudaError_t e);  // scan.cu
int bind_device(const void* ptr);                      // scan.cu

constexpr int kNormWarps = 8;        // rows per CTA
constexpr int kMaxPerLane = 32;      // dim <= 1024
constexpr int kNormBwdCtas = 8 * 148; // backward grid (CTAs stride over the rows)

static int64_t norm_bwd_blocks(int64_t rows) {
  const int64_t b = (rows + kNormWarps - 1) / kNormWarps;
  return b < kNormBwdCtas ? b : kNormBwdCtas;
}

template <typename T, int PER>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_fwd_kernel(ssm_norm_params_t p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kNormWarps + warp;
  if (row >= p.rows) return;
  const T* x = reinterpret_cast<const T*>(p.x) + row * p.dim;
  float v[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < p.dim ? Cvt<T>::to_f(x[c]) : 0.f;
    ss = fmaf(v[i], v[i], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / (float)p.dim + p.eps);
  T* y = reinterpret_cast<T*>(p.y) + row * p.dim;
  T* base = reinterpret_cast<T*>(p.res_base) + row * p.dim;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = lane + 32 * i;
    if (c < p.dim) {
      y[c] = Cvt<T>::from_f(v[i] * rstd * p.scale[c]);
      if (p.res_base) base[c] = Cvt<T>::from_f(v[i] + (p.res_bias ? p.res_bias[c] : 0.f));
    }
  }
  if (lane == 0) p.rstd[row] = rstd;
}

// dx = rstd * (g - x * rstd^2 * mean(g * x)) (+ dres),  g = dy * scale.
// Warps stride over the rows (fixed grid, fixed row assignment), accumulating
// sum dy * x * rstd per channel; each CTA writes one dscale partial.
template <typename T, int PER>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_bwd_kernel(ssm_norm_params_t p, float* dscale_part) {
  __shared__ float part[kNormWarps][32 * kMaxPerLane];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float ds[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) ds[i] = 0.f;
  const int64_t stride = (int64_t)gridDim.x * kNormWarps;
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + warp; row < p.rows; row += stride) {
    const T* x = reinterpret_cast<const T*>(p.x) + row * p.dim;
    const T* dy = reinterpret_cast<const T*>(p.dy) + row * p.dim;
    const float rstd = p.rstd[row];
    float xv[PER], gv[PER];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = lane + 32 * i;
      const bool ok = c < p.dim;
      xv[i] = ok ? Cvt<T>::to_f(x[c]) : 0.f;
      const float d = ok ? Cvt<T>::to_f(dy[c]) : 0.f;
      gv[i] = ok ? d * p.scale[c] : 0.f;
      dot = fmaf(gv[i], xv[i], dot);
      ds[i] = fmaf(d * xv[i], rstd, ds[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float k = rstd * rstd * dot / (float)p.dim;
    T* dx = reinterpret_cast<T*>(p.dx) + row * p.dim;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = lane + 32 * i;
      if (c < p.dim) {
        float g = rstd * (gv[i] - xv[i] * k);
        if (p.dres) g += Cvt<T>::to_f(reinterpret_cast<const T*>(p.dres)[row * p.dim + c]);
        dx[c] = Cvt<T>::from_f(g);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) part[warp][lane + 32 * i] = ds[i];
  __syncthreads();
  for (int c = threadIdx.x; c < p.dim; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kNormWarps; ++w) s += part[w][c];
    dscale_part[(int64_t)blockIdx.x * p.dim + c] = s;
  }
}

// dscale[c] = sum of the partials in block order
__global__ void rmsnorm_dscale_kernel(const float* part, int nparts, int dim, float* dscale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= dim) return;
  float s = 0.f;
  for (int i = 0; i < nparts; ++i) s += part[(int64_t)i * dim + c];
  dscale[c] = s;
}

static int check_norm(const ssm_norm_params_t* p) {
  if (!p) return SSM_ERR_NULL;
  if (p->rows < 0 || p->dim <= 0 || p->dim > 32 * kMaxPerLane) return SSM_ERR_SHAPE;
  if (p->dtype != SSM_F32 && p->dtype != SSM_BF16) return SSM_ERR_DTYPE;
  return SSM_OK;
}

template <typename T>
static void launch_norm_fwd(int per, dim3 grid, cudaStream_t s, const ssm_norm_params_t& p) {
  const dim3 block(32 * kNormWarps);
  if (per <= 8) rmsnorm_fwd_kernel<T, 8><<<grid, block, 0, s>>>(p);
  else if (per <= 16) rmsnorm_fwd_kernel<T, 16><<<grid, block, 0, s>>>(p);
  else rmsnorm_fwd_kernel<T, 32><<<grid, block, 0, s>>>(p);
}

template <typename T>
static void launch_norm_bwd(int per, dim3 grid, cudaStream_t s, const ssm_norm_params_t& p, float* part) {
  const dim3 block(32 * kNormWarps);
  if (per <= 8) rmsnorm_bwd_kernel<T, 8><<<grid, block, 0, s>>>(p, part);
  else if (per <= 16) rmsnorm_bwd_kernel<T, 16><<<grid, block, 0, s>>>(p, part);
  else rmsnorm_bwd_kernel<T, 32><<<grid, block, 0, s>>>(p, part);
}

}  // namespace ssm

using namespace ssm;

extern "C" {

size_t ssm_rmsnorm_workspace_bytes(const ssm_norm_params_t* p) {
  if (check_norm(p) || p->rows == 0) return 0;
  return (size_t)norm_bwd_blocks(p->rows) * p->dim * sizeof(float);
}

int ssm_rmsnorm_fwd(const ssm_norm_params_t* p, ssm_stream_t stream) {
  int st = check_norm(p);
  if (st) return st;
  if (p->rows == 0) return SSM_OK;
  if (!p->x || !p->scale || !p->y || !p->rstd) return SSM_ERR_NULL;
  st = bind_device(p->x);
  if (st) return st;
  const int per = (p->dim + 31) / 32;
  const dim3 grid((unsigned)((p->rows + kNormWarps - 1) / kNormWarps));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->dtype == SSM_BF16)
    launch_norm_fwd<__nv_bfloat16>(per, grid, s, *p);
  else
    launch_norm_fwd<float>(per, grid, s, *p);
  note_launches(1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SSM_OK : launch_error("launch rmsnorm_fwd_kernel", e);
}

int ssm_rmsnorm_bwd(const ssm_norm_params_t* p, ssm_stream_t stream) {
  int st = check_norm(p);
  if (st) return st;
  if (!p->dscale) return SSM_ERR_NULL;
  st = bind_device(p->dscale);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->rows == 0) {
    const cudaError_t e = cudaMemsetAsync(p->dscale, 0, (size_t)p->dim * sizeof(float), s);
    return e == cudaSuccess ? SSM_OK : launch_error("cudaMemsetAsync(dscale)", e);
  }
  if (!p->x || !p->scale || !p->rstd || !p->dy || !p->dx) return SSM_ERR_NULL;
  if (!p->workspace || p->workspace_bytes < ssm_rmsnorm_workspace_bytes(p)) return SSM_ERR_WORKSPACE;
  const int per = (p->dim + 31) / 32;
  const unsigned blocks = (unsigned)norm_bwd_blocks(p->rows);
  float* part = static_cast<float*>(p->workspace);
  if (p->dtype == SSM_BF16)
    launch_norm_bwd<__nv_bfloat16>(per, dim3(blocks), s, *p, part);
  else
    launch_norm_bwd<float>(per, dim3(blocks), s, *p, part);
  rmsnorm_dscale_kernel<<<(p->dim + 255) / 256, 256, 0, s>>>(part, (int)blocks, p->dim, p->dscale);
  note_launches(2);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SSM_OK : launch_error("launch rmsnorm_bwd_kernel", e);
}

}  // extern "C"
