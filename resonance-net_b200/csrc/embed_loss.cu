// Embedding gather / scatter, fused log-softmax cross-entropy, elementwise
// utilities.
//
// Reference: src/embedding.cu:6-47 (embedding), :71-92 (residual_add,
// scale_grads), :97-162 (cross_entropy_kernel: one CTA per token, loss by
// atomicAdd). Here the CE kernel is one warp per token with a deterministic
// two-level loss sum, and the 1/N dlogits scale of src/main.cpp:146 folded in.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

__global__ void embed_fwd_kernel(const int* __restrict__ tok, const float* __restrict__ table,
                                 float* __restrict__ out, int N, int V, int D, unsigned* err) {
  rnet_dev::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  int t = tok[warp];
  if (t < 0 || t >= V) {
    if (err && lane == 0) atomicOr(err, ERR_BAD_INDEX);
    t = 0;
  }
  const float4* src = reinterpret_cast<const float4*>(table + (size_t)t * D);
  float4* dst = reinterpret_cast<float4*>(out + (size_t)warp * D);
  for (int c = lane; c < D / 4; c += 32) dst[c] = src[c];
}

// Shared-memory privatised scatter: a CTA owns a 64-column slice of the table
// for all V rows and a range of tokens; one global atomic per (row, col, CTA).
constexpr int EB_COLS = 64;
__global__ void embed_bwd_kernel(const float* __restrict__ dout, const int* __restrict__ tok,
                                 float* __restrict__ dtable, int N, int V, int D,
                                 int tokens_per_cta) {
  rnet_dev::pdl_trigger();
  extern __shared__ float acc[];  // [V][EB_COLS]
  const int c0 = blockIdx.x * EB_COLS;
  const int n0 = blockIdx.y * tokens_per_cta;
  const int n1 = min(N, n0 + tokens_per_cta);
  for (int i = threadIdx.x; i < V * EB_COLS; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int n = n0 + warp; n < n1; n += nw) {
    const int t = tok[n];
    if (t < 0 || t >= V) continue;
    for (int c = lane; c < EB_COLS; c += 32) {
      const int col = c0 + c;
      if (col < D) atomicAdd(&acc[t * EB_COLS + c], dout[(size_t)n * D + col]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < V * EB_COLS; i += blockDim.x) {
    const int r = i / EB_COLS, c = c0 + i % EB_COLS;
    const float v = acc[i];
    if (c < D && v != 0.f) atomicAdd(&dtable[(size_t)r * D + c], v);
  }
}

// One warp per token row; V <= 32*32 values cached in registers.
constexpr int CE_MAXV = 32;
__global__ void ce_kernel(const float* __restrict__ logits, const int* __restrict__ tgt,
                          float* __restrict__ dl, float scale, float* __restrict__ part, int N,
                          int V, unsigned* err) {
  rnet_dev::pdl_trigger();
  __shared__ float wsum[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  float loss = 0.f;
  if (row < N) {
    const float* l = logits + (size_t)row * V;
    int t = tgt[row];
    if (t < 0 || t >= V) {
      if (err && lane == 0) atomicOr(err, ERR_BAD_INDEX);
      t = 0;
    }
    float v[CE_MAXV];
    float mx = -1e30f;
#pragma unroll
    for (int j = 0; j < CE_MAXV; ++j) {
      const int c = lane + 32 * j;
      v[j] = c < V ? l[c] : -1e30f;
      mx = fmaxf(mx, v[j]);
    }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < CE_MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < V) s += __expf(v[j] - mx);
    }
    s = warp_sum(s);
    const float ls = __logf(s);
    float* d = dl + (size_t)row * V;
#pragma unroll
    for (int j = 0; j < CE_MAXV; ++j) {
      const int c = lane + 32 * j;
      if (c < V) d[c] = (__expf(v[j] - mx - ls) - (c == t ? 1.f : 0.f)) * scale;
    }
    loss = -(l[t] - mx - ls);
  }
  if (lane == 0) wsum[warp] = loss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int j = 0; j < 8; ++j) a += wsum[j];
    part[blockIdx.x] = a;
  }
}

__global__ void sum_partials(const float* __restrict__ part, int n, float* __restrict__ out) {
  rnet_dev::pdl_trigger();
  __shared__ float sh[256];
  float a = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) a += part[i];
  sh[threadIdx.x] = a;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = sh[0];
}

__global__ void residual_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
  rnet_dev::pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    x[i] += y[i];
}
__global__ void scale_kernel(float* __restrict__ x, float a, size_t n) {
  rnet_dev::pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    x[i] *= a;
}
__global__ void add3_kernel(const float* __restrict__ a, const float* __restrict__ b,
                            const float* __restrict__ c, float* __restrict__ o, size_t n) {
  rnet_dev::pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    o[i] = a[i] + b[i] + c[i];
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                float* __restrict__ h, size_t n) {
  rnet_dev::pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float x = g[i];
    h[i] = silu_fast(x) * u[i];
  }
}

// SwiGLU backward pointwise step, in place over dgu = [dG | dU] ([N, 2F],
// row stride ld): on entry dG holds dH = dY W_down; on exit
//   dG = dH * u * silu'(g),  dU = dH * silu(g),
// silu'(g) = s + g s (1 - s), s = sigmoid(g) (reference src/swiglu_ffn.cu:23-40).
__device__ __forceinline__ void swiglu_grad1(float dh, float g, float u, float& dg, float& du) {
  const float sig = sigmoid_fast(g);
  const float dsilu = sig + g * sig * (1.0f - sig);
  dg = dh * u * dsilu;
  du = dh * (g * sig);
}

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

__global__ void swiglu_bwd_pointwise_v4(float* __restrict__ dgu, int ld,
                                        const float* __restrict__ G, const float* __restrict__ U,
                                        int N, int F, __nv_bfloat16* __restrict__ dgu16) {
  rnet_dev::pdl_trigger();
  const int F4 = F >> 2;
  const size_t n4 = (size_t)N * F4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / F4;
    const int c = (int)(i - r * F4) * 4;
    float4* pg = reinterpret_cast<float4*>(dgu + r * ld + c);
    float4* pu = reinterpret_cast<float4*>(dgu + r * ld + F + c);
    const float4 dh = *pg;
    const float4 g = *reinterpret_cast<const float4*>(G + r * F + c);
    const float4 u = *reinterpret_cast<const float4*>(U + r * F + c);
    float4 dg, du;
    swiglu_grad1(dh.x, g.x, u.x, dg.x, du.x);
    swiglu_grad1(dh.y, g.y, u.y, dg.y, du.y);
    swiglu_grad1(dh.z, g.z, u.z, dg.z, du.z);
    swiglu_grad1(dh.w, g.w, u.w, dg.w, du.w);
    if (dgu16) {
      st_bf16x4(dgu16 + r * ld + c, dg);
      st_bf16x4(dgu16 + r * ld + F + c, du);
    } else {
      *pg = dg;
      *pu = du;
    }
  }
}

__global__ void swiglu_bwd_pointwise_1(float* __restrict__ dgu, int ld,
                                       const float* __restrict__ G, const float* __restrict__ U,
                                       int N, int F, __nv_bfloat16* __restrict__ dgu16) {
  rnet_dev::pdl_trigger();
  const size_t n = (size_t)N * F;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / F;
    const int c = (int)(i - r * F);
    float dg, du;
    swiglu_grad1(dgu[r * ld + c], G[i], U[i], dg, du);
    if (dgu16) {
      dgu16[r * ld + c] = __float2bfloat16_rn(dg);
      dgu16[r * ld + F + c] = __float2bfloat16_rn(du);
    } else {
      dgu[r * ld + c] = dg;
      dgu[r * ld + F + c] = du;
    }
  }
}

int ew_grid(size_t n) {
  size_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

cudaError_t embed_fwd(const int* tok, const float* table, float* out, int N, int V, int D,
                      unsigned* err, cudaStream_t s) {
  if (N <= 0) return cudaSuccess;
  if (D % 4) return cudaErrorInvalidValue;
  embed_fwd_kernel<<<(N * 32 + 255) / 256, 256, 0, s>>>(tok, table, out, N, V, D, err);
  return launched();
}

cudaError_t embed_bwd(const float* dout, const int* tok, float* dtable, int N, int V, int D,
                      cudaStream_t s) {
  if (N <= 0) return cudaSuccess;
  const size_t smem = (size_t)V * EB_COLS * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(embed_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         200 * 1024);
    set = true;
  }
  const int cols = (D + EB_COLS - 1) / EB_COLS;
  int ctas = (148 * 2) / cols;
  if (ctas < 1) ctas = 1;
  int per = (N + ctas - 1) / ctas;
  if (per < 64) per = 64;
  dim3 grid(cols, (N + per - 1) / per);
  embed_bwd_kernel<<<grid, 512, smem, s>>>(dout, tok, dtable, N, V, D, per);
  return launched();
}

size_t ce_partials_floats(int N) { return (size_t)(N + 7) / 8 + 1; }

cudaError_t cross_entropy(const float* logits, const int* tgt, float* loss_sum, float* dl,
                          float scale, float* partials, int N, int V, unsigned* err,
                          cudaStream_t s) {
  if (V > 32 * CE_MAXV) return cudaErrorInvalidValue;
  const int blocks = (N + 7) / 8;
  if (N > 0) {
    ce_kernel<<<blocks, 256, 0, s>>>(logits, tgt, dl, scale, partials, N, V, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  sum_partials<<<1, 256, 0, s>>>(partials, blocks, loss_sum);
  return launched(N > 0 ? 2 : 1);
}

cudaError_t residual_add(float* x, const float* y, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  residual_kernel<<<ew_grid(n), 256, 0, s>>>(x, y, n);
  return launched();
}
cudaError_t scale(float* x, float a, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  scale_kernel<<<ew_grid(n), 256, 0, s>>>(x, a, n);
  return launched();
}
cudaError_t add3(const float* a, const float* b, const float* c, float* out, size_t n,
                 cudaStream_t s) {
  if (!n) return cudaSuccess;
  add3_kernel<<<ew_grid(n), 256, 0, s>>>(a, b, c, out, n);
  return launched();
}

cudaError_t swiglu_bwd_pointwise(float* dgu, int ld, const float* G, const float* U, int N, int F,
                                 cudaStream_t s, __nv_bfloat16* dgu16) {
  if (N <= 0 || F <= 0) return cudaSuccess;
  const bool v4 = (F % 4 == 0) && (ld % 4 == 0) &&
                  ((reinterpret_cast<uintptr_t>(dgu) | reinterpret_cast<uintptr_t>(G) |
                    reinterpret_cast<uintptr_t>(U) | reinterpret_cast<uintptr_t>(dgu16)) & 15) == 0;
  if (v4)
    swiglu_bwd_pointwise_v4<<<ew_grid((size_t)N * F / 4), 256, 0, s>>>(dgu, ld, G, U, N, F,
                                                                       dgu16);
  else
    swiglu_bwd_pointwise_1<<<ew_grid((size_t)N * F), 256, 0, s>>>(dgu, ld, G, U, N, F, dgu16);
  return launched();
}

cudaError_t silu_mul(const float* g, const float* u, float* h, size_t n, cudaStream_t s) {
  if (!n) return cudaSuccess;
  silu_mul_kernel<<<ew_grid(n), 256, 0, s>>>(g, u, h, n);
  return launched();
}

}  // namespace rnet_k
