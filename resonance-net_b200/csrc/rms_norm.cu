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
#include "status.h"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int WARPS = 8;

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

template <int VPL>
__global__ void __launch_bounds__(WARPS * 32)
    rms_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                   float* __restrict__ y, float* __restrict__ rinv, int rows, int D, float eps,
                   float* __restrict__ xcopy, __nv_bfloat16* __restrict__ y16) {
  rnet_dev::pdl_trigger();
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
    if (xcopy) {
      float4* cr = reinterpret_cast<float4*>(xcopy + (size_t)row * D);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < nv) cr[c] = v[j];
      }
    }
    ss = warp_sum(ss);
    const float ri = rsqrtf(ss / (float)D + eps);
    if (lane == 0 && rinv) rinv[row] = ri;
    if (y || y16) {
      float4* yr = reinterpret_cast<float4*>(y + (size_t)row * D);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < nv) {
          const float4 g = w4[c];
          const float4 o = make_float4(v[j].x * ri * g.x, v[j].y * ri * g.y, v[j].z * ri * g.z,
                                       v[j].w * ri * g.w);
          if (y) yr[c] = o;
          if (y16) st_bf16x4(y16 + (size_t)row * D + 4 * c, o);
        }
      }
    }
  }
}

template <int VPL>
__global__ void __launch_bounds__(WARPS * 32)
    rms_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const float* __restrict__ w, const float* __restrict__ rinv,
                   float* __restrict__ dx, float* __restrict__ dw, int rows, int D, int mode,
                   __nv_bfloat16* __restrict__ dx16) {
  rnet_dev::pdl_trigger();
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
        if (dx16) st_bf16x4(dx16 + (size_t)row * D + 4 * c, o);
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

// Backward for wide rows (D > 512, e.g. 2048): a row per CTA of RB_THREADS
// threads (VPT float4 per thread) instead of a row per warp, which would
// need 16 float4 per lane per array and spill. The row's dot product is a
// block reduction through a double-buffered shared array (one barrier per
// row); each thread keeps the dw partial of its fixed columns in registers
// over all rows of the CTA and flushes it once with atomics.
constexpr int RB_THREADS = 256;

template <int VPT>
__global__ void __launch_bounds__(RB_THREADS)
    rms_bwd_rowblock_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                            const float* __restrict__ w, const float* __restrict__ rinv,
                            float* __restrict__ dx, float* __restrict__ dw, int rows, int D,
                            int mode, __nv_bfloat16* __restrict__ dx16) {
  rnet_dev::pdl_trigger();
  __shared__ float red[2][RB_THREADS / 32];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nv = D >> 2;
  const float invD = 1.0f / (float)D;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[VPT], acc[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = t + RB_THREADS * j;
    wv[j] = c < nv ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int par = 0;
  for (int row = blockIdx.x; row < rows; row += gridDim.x, par ^= 1) {
    const float4* dyr = reinterpret_cast<const float4*>(dy + (size_t)row * D);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    float4* dxr = reinterpret_cast<float4*>(dx + (size_t)row * D);
    const float ri = rinv[row];
    float4 g[VPT], xh[VPT], prev[VPT];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = t + RB_THREADS * j;
      if (c < nv) {
        const float4 a = dyr[c], b = xr[c], ww = wv[j];
        prev[j] = mode == 1 ? dxr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        g[j] = a;
        xh[j] = make_float4(b.x * ri, b.y * ri, b.z * ri, b.w * ri);
        dot += a.x * ww.x * xh[j].x + a.y * ww.y * xh[j].y + a.z * ww.z * xh[j].z +
               a.w * ww.w * xh[j].w;
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) red[par][warp] = dot;
    __syncthreads();
    dot = 0.f;
#pragma unroll
    for (int k = 0; k < RB_THREADS / 32; ++k) dot += red[par][k];
    dot *= invD;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = t + RB_THREADS * j;
      if (c < nv) {
        const float4 ww = wv[j];
        float4 o = make_float4(ri * (g[j].x * ww.x - xh[j].x * dot),
                               ri * (g[j].y * ww.y - xh[j].y * dot),
                               ri * (g[j].z * ww.z - xh[j].z * dot),
                               ri * (g[j].w * ww.w - xh[j].w * dot));
        o.x += prev[j].x; o.y += prev[j].y; o.z += prev[j].z; o.w += prev[j].w;
        dxr[c] = o;
        if (dx16) st_bf16x4(dx16 + (size_t)row * D + 4 * c, o);
        acc[j].x += g[j].x * xh[j].x;
        acc[j].y += g[j].y * xh[j].y;
        acc[j].z += g[j].z * xh[j].z;
        acc[j].w += g[j].w * xh[j].w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = t + RB_THREADS * j;
    if (c < nv) {
      atomicAdd(&dw[4 * c], acc[j].x);
      atomicAdd(&dw[4 * c + 1], acc[j].y);
      atomicAdd(&dw[4 * c + 2], acc[j].z);
      atomicAdd(&dw[4 * c + 3], acc[j].w);
    }
  }
}

// Backward for D <= STAGED_MAX_D: persistent CTAs walk groups of WARPS rows
// (one row per warp); the dy / x (/ dx when accumulating) rows of the next
// group are copied global -> shared while the current group is computed, so
// loads stay in flight through the reductions and stores. A group's rows are
// contiguous: thread 0 moves each array with one bulk copy (completion on the
// stage's mbarrier), and the other threads do no address arithmetic.
constexpr int STAGED_MAX_D = 512;

// Untiled bulk copy global -> shared (16-byte aligned, size % 16 == 0), no
// multicast; completes `bytes` on the mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(void* smem, const void* gmem, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int VPL>
__global__ void __launch_bounds__(WARPS * 32, 2)
    rms_bwd_staged_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                          const float* __restrict__ w, const float* __restrict__ rinv,
                          float* __restrict__ dx, float* __restrict__ dw, int rows, int D,
                          int mode, unsigned* err, __nv_bfloat16* __restrict__ dx16) {
  rnet_dev::pdl_trigger();
  // [2 stages][3 arrays][WARPS rows][D]
  extern __shared__ __align__(16) float sbuf[];
  __shared__ uint64_t full[2];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = D >> 2;
  const int narr = mode == 1 ? 3 : 2;
  auto slot = [&](int st, int arr, int wr) {
    return sbuf + ((size_t)(st * 3 + arr) * WARPS + wr) * D;
  };
  const int ngroups = (rows + WARPS - 1) / WARPS;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Stage group g into stage st (thread 0: one bulk copy per array). After a
  // timed-out wait (abort_flag) nothing new is issued; thread 0 counts the
  // copies issued and consumed per stage so the abort path can drain them.
  int issued[2] = {0, 0}, consumed[2] = {0, 0};
  auto stage = [&](int g, int st) {
    if (threadIdx.x == 0 && g < ngroups && !abort_flag) {
      ++issued[st];
      const int r0 = g * WARPS;
      const int nr = rows - r0 < WARPS ? rows - r0 : WARPS;
      const uint32_t bytes = (uint32_t)nr * D * 4;
      mbar_arrive_expect_tx(&full[st], narr * bytes);
      bulk_load(slot(st, 0, 0), dy + (size_t)r0 * D, bytes, &full[st]);
      bulk_load(slot(st, 1, 0), x + (size_t)r0 * D, bytes, &full[st]);
      if (narr == 3) bulk_load(slot(st, 2, 0), dx + (size_t)r0 * D, bytes, &full[st]);
    }
  };
  float4 acc[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    wv[j] = c < nv ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float invD = 1.0f / (float)D;
  int st = 0, it = 0;
  bool ok = true;  // a failed (timed-out) wait skips the compute, not the barriers
  stage(blockIdx.x, 0);
  for (int g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
    stage(g + gridDim.x, st ^ 1);
    ok = ok && mbar_wait(&full[st], (it >> 1) & 1, err, &abort_flag);
    if (ok) ++consumed[st];
    const int row = g * WARPS + warp;
    if (ok && row < rows) {
      const float4* dyr = reinterpret_cast<const float4*>(slot(st, 0, warp));
      const float4* xr = reinterpret_cast<const float4*>(slot(st, 1, warp));
      const float4* pr = reinterpret_cast<const float4*>(slot(st, 2, warp));
      const float ri = rinv[row];
      float4 gv[VPL], xh[VPL];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < nv) {
          const float4 a = dyr[c], b = xr[c], ww = wv[j];
          gv[j] = a;
          xh[j] = make_float4(b.x * ri, b.y * ri, b.z * ri, b.w * ri);
          dot += a.x * ww.x * xh[j].x + a.y * ww.y * xh[j].y + a.z * ww.z * xh[j].z +
                 a.w * ww.w * xh[j].w;
        }
      }
      dot = warp_sum(dot) * invD;
      float4* dxr = reinterpret_cast<float4*>(dx + (size_t)row * D);
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int c = lane + 32 * j;
        if (c < nv) {
          const float4 ww = wv[j];
          float4 o = make_float4(ri * (gv[j].x * ww.x - xh[j].x * dot),
                                 ri * (gv[j].y * ww.y - xh[j].y * dot),
                                 ri * (gv[j].z * ww.z - xh[j].z * dot),
                                 ri * (gv[j].w * ww.w - xh[j].w * dot));
          if (mode == 1) {
            const float4 p = pr[c];
            o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
          }
          dxr[c] = o;
          if (dx16) st_bf16x4(dx16 + (size_t)row * D + 4 * c, o);
          acc[j].x += gv[j].x * xh[j].x;
          acc[j].y += gv[j].y * xh[j].y;
          acc[j].z += gv[j].z * xh[j].z;
          acc[j].w += gv[j].w * xh[j].w;
        }
      }
    }
    __syncthreads();  // stage `st` is refilled next iteration
    st ^= 1;
  }
  __syncthreads();
  if (abort_flag) {
    // Failure path: wait (bounded) for the bulk copies still in flight into
    // shared memory, then leave dw untouched; the error word reports it.
    if (threadIdx.x == 0) {
      volatile int no_abort = 0;
      for (int b = 0; b < 2; ++b)
        while (consumed[b] < issued[b] &&
               mbar_wait_for(&full[b], consumed[b] & 1, nullptr, &no_abort, RNET_WAIT_TIMEOUT_NS))
          ++consumed[b];
    }
    return;
  }
  // per-warp partials (reusing the staging buffer), fixed-order sum over warps
  float* sdw = sbuf;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) reinterpret_cast<float4*>(sdw + (size_t)warp * D)[c] = acc[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float sum = 0.f;
    for (int k = 0; k < WARPS; ++k) sum += sdw[(size_t)k * D + i];
    atomicAdd(&dw[i], sum);
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
                  float eps, cudaStream_t s, float* xcopy, __nv_bfloat16* y16) {
  const int need = (rows + WARPS - 1) / WARPS;
  const int cap = sm_count() * 8;
  rms_fwd_kernel<VPL><<<need < cap ? need : cap, WARPS * 32, 0, s>>>(x, w, y, rinv, rows, D, eps,
                                                                          xcopy, y16);
  return launched();
}

template <int VPL>
cudaError_t bwd_t(const float* dy, const float* x, const float* w, const float* rinv, float* dx,
                  float* dw, int rows, int D, int mode, cudaStream_t s, __nv_bfloat16* dx16) {
  if constexpr (VPL * 128 <= STAGED_MAX_D) {
    const size_t smem = (size_t)2 * 3 * WARPS * D * sizeof(float);
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(rms_bwd_staged_kernel<VPL>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)((size_t)2 * 3 * WARPS * STAGED_MAX_D * sizeof(float)));
      set = true;
    }
    const int ngroups = (rows + WARPS - 1) / WARPS;
    int grid = sm_count() * 2;  // two CTAs per SM (2 x 96 KB at D = 512)
    if (grid > ngroups) grid = ngroups;
    rms_bwd_staged_kernel<VPL><<<grid, WARPS * 32, smem, s>>>(dy, x, w, rinv, dx, dw, rows, D,
                                                              mode,
                                                              rnet_status::device_error_word(),
                                                              dx16);
    return launched();
  }
  if constexpr (VPL >= 8) {
    // wide rows: a row per 256-thread CTA (VPL / 8 float4 per thread)
    constexpr int VPT = VPL / 8;
    int grid = sm_count() * 4;
    if (grid > rows) grid = rows;
    rms_bwd_rowblock_kernel<VPT><<<grid, RB_THREADS, 0, s>>>(dy, x, w, rinv, dx, dw, rows, D,
                                                             mode, dx16);
    return launched();
  }
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
  rms_bwd_kernel<VPL><<<grid, WARPS * 32, smem, s>>>(dy, x, w, rinv, dx, dw, rows, D, mode, dx16);
  return launched();
}

}  // namespace

cudaError_t rms_norm_fwd(const float* x, const float* w, float* y, float* rinv, int rows, int D,
                         float eps, cudaStream_t s, float* xcopy, __nv_bfloat16* y16) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 2048) return cudaErrorInvalidValue;
  const int vpl = (D + 127) / 128;
  if (vpl <= 1) return fwd_t<1>(x, w, y, rinv, rows, D, eps, s, xcopy, y16);
  if (vpl <= 2) return fwd_t<2>(x, w, y, rinv, rows, D, eps, s, xcopy, y16);
  if (vpl <= 4) return fwd_t<4>(x, w, y, rinv, rows, D, eps, s, xcopy, y16);
  if (vpl <= 8) return fwd_t<8>(x, w, y, rinv, rows, D, eps, s, xcopy, y16);
  return fwd_t<16>(x, w, y, rinv, rows, D, eps, s, xcopy, y16);
}

cudaError_t rms_norm_bwd(const float* dy, const float* x, const float* w, const float* rinv,
                         float* dx, float* dw, int rows, int D, int mode, cudaStream_t s,
                         __nv_bfloat16* dx16) {
  if (rows <= 0) return cudaSuccess;
  if (D % 4 != 0 || D > 2048) return cudaErrorInvalidValue;
  const int vpl = (D + 127) / 128;
  if (vpl <= 1) return bwd_t<1>(dy, x, w, rinv, dx, dw, rows, D, mode, s, dx16);
  if (vpl <= 2) return bwd_t<2>(dy, x, w, rinv, dx, dw, rows, D, mode, s, dx16);
  if (vpl <= 4) return bwd_t<4>(dy, x, w, rinv, dx, dw, rows, D, mode, s, dx16);
  if (vpl <= 8) return bwd_t<8>(dy, x, w, rinv, dx, dw, rows, D, mode, s, dx16);
  return bwd_t<16>(dy, x, w, rinv, dx, dw, rows, D, mode, s, dx16);
}

}  // namespace rnet_k
