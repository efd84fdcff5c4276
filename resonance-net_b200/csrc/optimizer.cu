// Global-norm gradient clipping + SGD over the flat parameter buffer, entirely
// on the device (no host round trip).
//
// Reference: src/resonance_net.cpp:551-663 — lr /= world_size under DDP,
// ||g|| from one cublasSdot per tensor (each a host sync), clip against
// ||g|| / world_size, then one cublasSaxpy(-lr) per tensor. Here: a fixed-grid
// double-precision sum of squares, a single-block finalisation that computes
// the effective learning rate on the device, and one vectorised update pass.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {

namespace {

constexpr int NORM_BLOCKS = 592;  // 4 x 148, fixed so the reduction order is fixed

__global__ void sumsq_kernel(const float* __restrict__ g, size_t n, double* __restrict__ part) {
  rnet_dev::pdl_trigger();
  __shared__ double sh[256];
  double a = 0.0;
  const size_t n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = g4[i];
    a += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) a += (double)g[i] * g[i];
  sh[threadIdx.x] = a;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

__global__ void finalize_kernel(const double* __restrict__ part, int nparts, float lr,
                                float clip, int world, float* __restrict__ lr_out,
                                float* __restrict__ norm_out) {
  rnet_dev::pdl_trigger();
  __shared__ double sh[256];
  double a = 0.0;
  for (int i = threadIdx.x; i < nparts; i += 256) a += part[i];
  sh[threadIdx.x] = a;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double norm = sqrt(sh[0]);
    float l = lr;
    if (world > 1) l /= (float)world;
    const double avg = norm / (world > 1 ? world : 1);
    if (clip > 0.f && avg > clip) l = (float)(l * (clip / avg));
    *lr_out = l;
    if (norm_out) *norm_out = (float)norm;
  }
}

// Optional extensions (off by default, so the step is the reference's plain
// SGD): weight decay wd adds wd * p to the gradient; momentum mu keeps a
// velocity v = mu * v + g (+ wd * p) and steps along it.
__device__ __forceinline__ float upd1(float p, float g, float* v, float neg, float mu, float wd) {
  float d = g + wd * p;
  if (v) {
    d += mu * *v;
    *v = d;
  }
  return p + neg * d;
}

__global__ void update_kernel(float* __restrict__ p, const float* __restrict__ g, size_t n,
                              const float* __restrict__ lr_ptr, __nv_bfloat16* __restrict__ p16,
                              float* __restrict__ vel, float mu, float wd) {
  rnet_dev::pdl_trigger();
  const float neg = -*lr_ptr;
  const size_t n4 = n / 4;
  float4* p4 = reinterpret_cast<float4*>(p);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  float4* v4 = reinterpret_cast<float4*>(vel);
  const bool plain = vel == nullptr && wd == 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    float4 a = p4[i];
    const float4 b = g4[i];
    if (plain) {
      a.x += neg * b.x; a.y += neg * b.y; a.z += neg * b.z; a.w += neg * b.w;
    } else {
      float4 v = vel ? v4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      a.x = upd1(a.x, b.x, vel ? &v.x : nullptr, neg, mu, wd);
      a.y = upd1(a.y, b.y, vel ? &v.y : nullptr, neg, mu, wd);
      a.z = upd1(a.z, b.z, vel ? &v.z : nullptr, neg, mu, wd);
      a.w = upd1(a.w, b.w, vel ? &v.w : nullptr, neg, mu, wd);
      if (vel) v4[i] = v;
    }
    p4[i] = a;
    if (p16) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&lo);
      u.y = *reinterpret_cast<const uint32_t*>(&hi);
      reinterpret_cast<uint2*>(p16)[i] = u;
    }
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
      p[i] = upd1(p[i], g[i], vel ? vel + i : nullptr, neg, mu, wd);
      if (p16) p16[i] = __float2bfloat16_rn(p[i]);
    }
}

__global__ void to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                               size_t n) {
  rnet_dev::pdl_trigger();
  const size_t n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = x4[i];
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&lo);
    u.y = *reinterpret_cast<const uint32_t*>(&hi);
    reinterpret_cast<uint2*>(y)[i] = u;
  }
  if (blockIdx.x == 0)
    for (size_t i = n4 * 4 + threadIdx.x; i < n; i += blockDim.x) y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void from_bf16_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y,
                                 size_t n) {
  rnet_dev::pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

}  // namespace

size_t sgd_scratch_floats() { return 2 * NORM_BLOCKS + 8; }

cudaError_t to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 7))
    return cudaErrorInvalidValue;
  size_t grid = (n / 4 + 255) / 256;
  if (grid > 148 * 8) grid = 148 * 8;
  if (grid < 1) grid = 1;
  to_bf16_kernel<<<(unsigned)grid, 256, 0, s>>>(x, y, n);
  return launched();
}

cudaError_t from_bf16(const __nv_bfloat16* x, float* y, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  size_t grid = (n + 255) / 256;
  if (grid > 148 * 8) grid = 148 * 8;
  from_bf16_kernel<<<(unsigned)grid, 256, 0, s>>>(x, y, n);
  return launched();
}

cudaError_t sgd_clip_step(float* params, const float* grads, size_t n, float lr, float clip,
                          int world, float* scratch, float* norm_out, cudaStream_t s,
                          __nv_bfloat16* params16, float* velocity, float momentum,
                          float weight_decay) {
  if (!n) return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(grads)) & 15)
    return cudaErrorInvalidValue;
  double* part = reinterpret_cast<double*>(scratch);
  float* lr_dev = scratch + 2 * NORM_BLOCKS;
  sumsq_kernel<<<NORM_BLOCKS, 256, 0, s>>>(grads, n, part);
  finalize_kernel<<<1, 256, 0, s>>>(part, NORM_BLOCKS, lr, clip, world, lr_dev, norm_out);
  update_kernel<<<148 * 8, 256, 0, s>>>(params, grads, n, lr_dev, params16, velocity, momentum,
                                        weight_decay);
  return launched(3);
}

}  // namespace rnet_k
