// RMSNorm forward / backward, one warp per row, 128-bit loads, the row kept
// in registers between the reduction and the output pass.
//
// Reference: src/rms_norm.cu:8-47 (forward), :52-90 (backward). The backward
// here also folds the residual add of src/resonance_net.cpp:488/508/526/543
// (mode 1) and replaces the per-element atomicAdd into dw by per-CTA partial
// sums (one atomic per column per CTA).
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int WARPS = 8;
constexpr int MAXV = 16;  // float4 per lane -> D <= 2048

__global__ void __launch_bounds__(WARPS * 32)
    rms_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                   float* __restrict__ y, float* __restrict__ rinv, int rows, int D, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 2;  // float4 per row
  for (int row = blockIdx.x * WARPS + warp; row < rows; row += gridDim.x * WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    float4 v[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        v[j] = xr[c];
        ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      }
    }
    ss = warp_sum(ss);
    const float ri = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rinv) rinv[row] = ri;
    if (y) {
      float4* yr = reinterpret_cast<float4*>(y + (size_t)row * D);
      const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
      for (int j = 0; j < MAXV; ++j) {
        const int c = lane + 32 * j;
        if (c < nv) {
          const float4 g = w4[c];
          yr[c] = make_float4(v[j].x * ri * g.x, v[j].y * ri * g.y, v[j].z * ri * g.z,
                              v[j].w * ri * g.w);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(WARPS * 32)
    rms_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const float* __restrict__ w, const float* __restrict__ rinv,
                   float* __restrict__ dx, float* __restrict__ dw, int rows, int D, int mode) {
  extern __shared__ float sdw[];  // [D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 2;
  for (int i = threadIdx.x; i < D; i += blockDim.x) sdw[i] = 0.f;
  float4 acc[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float invD = 1.0f / (float)D;
  for (int row = blockIdx.x * WARPS + warp; row < rows; row += gridDim.x * WARPS) {
    const float4* dyr = reinterpret_cast<const float4*>(dy + (size_t)row * D);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    const float ri = rinv[row];
    float4 g[MAXV], xh[MAXV];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 a = dyr[c], b = xr[c], ww = w4[c];
        g[j] = a;
        xh[j] = make_float4(b.x * ri, b.y * ri, b.z * ri, b.w * ri);
        dot += a.x * ww.x * xh[j].x + a.y * ww.y * xh[j].y + a.z * ww.z * xh[j].z +
               a.w * ww.w * xh[j].w;
      }
    }
    dot = warp_sum(dot) * invD;
    float4* dxr = reinterpret_cast<float4*>(dx + (size_t)row * D);
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 ww = w4[c];
        float4 o = make_float4(ri * (g[j].x * ww.x - xh[j].x * dot),
                               ri * (g[j].y * ww.y - xh[j].y * dot),
                               ri * (g[j].z * ww.z - xh[j].z * dot),
                               ri * (g[j].w * ww.w - xh[j].w * dot));
        if (mode == 1) {
          const float4 p = dxr[c];
          o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
        }
        dxr[c] = o;
        acc[j].x += g[j].x * xh[j].x;
        acc[j].y += g[j].y * xh[j].y;
        acc[j].z += g[j].z * xh[j].z;
        acc[j].w += g[j].w * xh[j].w;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      atomicAdd(&sdw[4 * c + 0], acc[j].x);
      atomicAdd(&sdw[4 * c + 1], acc[j].y);
      atomicAdd(&sdw[4 * c + 2], acc[j].z);
      atomicAdd(&sdw[4 * c + 3], acc[j].w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

int grid_for_rows(int rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int need = (rows + WARPS - 1) / WARPS;
  const int cap = sms * 8;
  return need < cap ? (need > 0 ? need : 1) : cap;
}

}  // namespace

cudaError_t rms_norm_fwd(const float* x, const float* w, float* y, float* rinv, int rows, int D,
                         float eps, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 4 * 32 * MAXV) return cudaErrorInvalidValue;
  rms_fwd_kernel<<<grid_for_rows(rows), WARPS * 32, 0, s>>>(x, w, y, rinv, rows, D, eps);
  return launched();
}

cudaError_t rms_norm_bwd(const float* dy, const float* x, const float* w, const float* rinv,
                         float* dx, float* dw, int rows, int D, int mode, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 4 * 32 * MAXV) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int grid = (rows + WARPS * 4 - 1) / (WARPS * 4);  // >= 4 rows per warp
  if (grid > sms * 2) grid = sms * 2;
  if (grid < 1) grid = 1;
  rms_bwd_kernel<<<grid, WARPS * 32, D * sizeof(float), s>>>(dy, x, w, rinv, dx, dw, rows, D,
                                                             mode);
  return launched();
}

}  // namespace rnet_k
