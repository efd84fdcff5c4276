// RMSNorm forward / backward, one warp per row, 128-bit loads, the row kept
// in registers between the reduction and the output pass.
//
// Reference: src/rms_norm.cu:8-47 (forward), :52-90 (backward). The backward
// here also folds the residual add of src/resonance_net.cpp:488/508/526/543
// (mode 1) and replaces the per-element atomicAdd into dw by per-CTA partial
// sums (one atomic per column per CTA).
//
// Templated on VPL = float4 vectors per lane per row (D <= 128 * VPL, tail
// lanes masked) so the row fits in registers without spilling and occupancy
// stays high (D = 512 -> VPL 4).
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int WARPS = 8;

template <int VPL>
__global__ void __launch_bounds__(WARPS * 32)
    rms_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                   float* __restrict__ y, float* __restrict__ rinv, int rows, int D, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int row = blockIdx.x * WARPS + warp; row < rows; row += gridDim.x * WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    float4 v[VPL];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      v[j] = c < nv ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
    ss = warp_sum(ss);
    const float ri = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rinv) rinv[row] = ri;
    if (y) {
      float4* yr = reinterpret_cast<float4*>(y + (size_t)row * D);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
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

template <int VPL>
__global__ void __launch_bounds__(WARPS * 32)
    rms_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const float* __restrict__ w, const float* __restrict__ rinv,
                   float* __restrict__ dx, float* __restrict__ dw, int rows, int D, int mode) {
  extern __shared__ float sdw[];  // [WARPS][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 2;
  float4 acc[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float invD = 1.0f / (float)D;
  for (int row = blockIdx.x * WARPS + warp; row < rows; row += gridDim.x * WARPS) {
    const float4* dyr = reinterpret_cast<const float4*>(dy + (size_t)row * D);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    float4* dxr = reinterpret_cast<float4*>(dx + (size_t)row * D);
    const float ri = rinv[row];
    float4 g[VPL], xh[VPL], prev[VPL];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 a = dyr[c], b = xr[c], ww = w4[c];
        prev[j] = mode == 1 ? dxr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        g[j] = a;
        xh[j] = make_float4(b.x * ri, b.y * ri, b.z * ri, b.w * ri);
        dot += a.x * ww.x * xh[j].x + a.y * ww.y * xh[j].y + a.z * ww.z * xh[j].z +
               a.w * ww.w * xh[j].w;
      }
    }
    dot = warp_sum(dot) * invD;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < nv) {
        const float4 ww = w4[c];
        float4 o = make_float4(ri * (g[j].x * ww.x - xh[j].x * dot),
                               ri * (g[j].y * ww.y - xh[j].y * dot),
                               ri * (g[j].z * ww.z - xh[j].z * dot),
                               ri * (g[j].w * ww.w - xh[j].w * dot));
        o.x += prev[j].x; o.y += prev[j].y; o.z += prev[j].z; o.w += prev[j].w;
        dxr[c] = o;
        acc[j].x += g[j].x * xh[j].x;
        acc[j].y += g[j].y * xh[j].y;
        acc[j].z += g[j].z * xh[j].z;
        acc[j].w += g[j].w * xh[j].w;
      }
    }
  }
  // per-warp partials to shared memory, then a fixed-order sum over warps
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) reinterpret_cast<float4*>(sdw + (size_t)warp * D)[c] = acc[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < WARPS; ++k) s += sdw[(size_t)k * D + i];
    atomicAdd(&dw[i], s);
  }
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <int VPL>
cudaError_t fwd_t(const float* x, const float* w, float* y, float* rinv, int rows, int D,
                  float eps, cudaStream_t s) {
  const int need = (rows + WARPS - 1) / WARPS;
  const int cap = sm_count() * 8;
  rms_fwd_kernel<VPL><<<need < cap ? need : cap, WARPS * 32, 0, s>>>(x, w, y, rinv, rows, D, eps);
  return launched();
}

template <int VPL>
cudaError_t bwd_t(const float* dy, const float* x, const float* w, const float* rinv, float* dx,
                  float* dw, int rows, int D, int mode, cudaStream_t s) {
  // >= 4 rows per warp so the dw partial flush is amortised
  int grid = (rows + WARPS * 4 - 1) / (WARPS * 4);
  const int cap = sm_count() * 6;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  const size_t smem = (size_t)WARPS * D * sizeof(float);
  if (smem > 48 * 1024) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(rms_bwd_kernel<VPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      set = true;
    }
  }
  rms_bwd_kernel<VPL><<<grid, WARPS * 32, smem, s>>>(dy, x, w, rinv, dx, dw, rows, D, mode);
  return launched();
}

}  // namespace

cudaError_t rms_norm_fwd(const float* x, const float* w, float* y, float* rinv, int rows, int D,
                         float eps, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 2048) return cudaErrorInvalidValue;
  const int vpl = (D + 127) / 128;
  if (vpl <= 1) return fwd_t<1>(x, w, y, rinv, rows, D, eps, s);
  if (vpl <= 2) return fwd_t<2>(x, w, y, rinv, rows, D, eps, s);
  if (vpl <= 4) return fwd_t<4>(x, w, y, rinv, rows, D, eps, s);
  if (vpl <= 8) return fwd_t<8>(x, w, y, rinv, rows, D, eps, s);
  return fwd_t<16>(x, w, y, rinv, rows, D, eps, s);
}

cudaError_t rms_norm_bwd(const float* dy, const float* x, const float* w, const float* rinv,
                         float* dx, float* dw, int rows, int D, int mode, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 2048) return cudaErrorInvalidValue;
  const int vpl = (D + 127) / 128;
  if (vpl <= 1) return bwd_t<1>(dy, x, w, rinv, dx, dw, rows, D, mode, s);
  if (vpl <= 2) return bwd_t<2>(dy, x, w, rinv, dx, dw, rows, D, mode, s);
  if (vpl <= 4) return bwd_t<4>(dy, x, w, rinv, dx, dw, rows, D, mode, s);
  if (vpl <= 8) return bwd_t<8>(dy, x, w, rinv, dx, dw, rows, D, mode, s);
  return bwd_t<16>(dy, x, w, rinv, dx, dw, rows, D, mode, s);
}

}  // namespace rnet_k
