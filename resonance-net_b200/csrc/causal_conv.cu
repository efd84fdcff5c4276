// Multi-scale depthwise causal convolution (k = 3, 7, 15) fused into one pass.
//
// Reference: src/causal_conv.cu:9-30 (one depthwise kernel launched per scale),
// :33-39 + :61-71 (sum3 into the c3 slot), :85-130 and :150-187 (data and
// weight gradients, the weight gradient on only K blocks). Here one thread
// owns one channel over a 32-step time chunk, holds the 46-sample window
// (14-step causal halo) in registers and produces all three scales; the weight
// gradient is a two-level deterministic reduction over (batch, chunk).
//
// Per-scale accumulation order matches the reference (sum += x*w over taps in
// increasing k, zero left padding), and S = (c3 + c7) + c15 as its sum3.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {

namespace {

constexpr int TC = 32;    // time steps per thread
constexpr int HALO = 14;  // max kernel size - 1
constexpr int CPB = 128;  // channels per block
constexpr int MAX_PARTS = 192;

__global__ void __launch_bounds__(CPB)
    conv_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w3,
                    const float* __restrict__ w7, const float* __restrict__ w15,
                    float* __restrict__ S, float* __restrict__ Sq, float* __restrict__ c7o,
                    float* __restrict__ c15o, int T, int D, int nchunks) {
  const int d = blockIdx.x * CPB + threadIdx.x;
  if (d >= D) return;
  const int b = blockIdx.y / nchunks;
  const int t0 = (blockIdx.y % nchunks) * TC;
  const float* xb = x + (size_t)b * T * D + d;
  float win[TC + HALO];
#pragma unroll
  for (int i = 0; i < TC + HALO; ++i) {
    const int t = t0 - HALO + i;
    win[i] = (t >= 0 && t < T) ? xb[(size_t)t * D] : 0.0f;
  }
  float a3[3], a7[7], a15[15];
#pragma unroll
  for (int k = 0; k < 3; ++k) a3[k] = w3[k * D + d];
#pragma unroll
  for (int k = 0; k < 7; ++k) a7[k] = w7[k * D + d];
#pragma unroll
  for (int k = 0; k < 15; ++k) a15[k] = w15[k * D + d];
  const size_t base = (size_t)b * T * D + d;
#pragma unroll
  for (int i = 0; i < TC; ++i) {
    const int t = t0 + i;
    if (t >= T) break;
    // output t uses x[t-(K-1)+k] = win[i + HALO - (K-1) + k]
    float s3 = 0.f, s7 = 0.f, s15 = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) s3 += win[i + HALO - 2 + k] * a3[k];
#pragma unroll
    for (int k = 0; k < 7; ++k) s7 += win[i + HALO - 6 + k] * a7[k];
#pragma unroll
    for (int k = 0; k < 15; ++k) s15 += win[i + k] * a15[k];
    const float sum = s3 + s7 + s15;
    const size_t o = base + (size_t)t * D;
    S[o] = sum;
    if (Sq) Sq[o] = sum + s7 + s15;
    if (c7o) c7o[o] = s7;
    if (c15o) c15o[o] = s15;
  }
}

// Data + weight gradient. Block (channel group, part p) loops over work
// items (b, chunk) = p, p + nparts, ...
__global__ void __launch_bounds__(CPB)
    conv_bwd_kernel(const float* __restrict__ dS, const float* __restrict__ x,
                    const float* __restrict__ w3, const float* __restrict__ w7,
                    const float* __restrict__ w15, float* __restrict__ dx,
                    float* __restrict__ parts, int B, int T, int D, int nchunks, int nparts,
                    int accumulate) {
  const int d = blockIdx.x * CPB + threadIdx.x;
  if (d >= D) return;
  float a3[3], a7[7], a15[15];
#pragma unroll
  for (int k = 0; k < 3; ++k) a3[k] = w3[k * D + d];
#pragma unroll
  for (int k = 0; k < 7; ++k) a7[k] = w7[k * D + d];
#pragma unroll
  for (int k = 0; k < 15; ++k) a15[k] = w15[k * D + d];
  float g3[3] = {0, 0, 0}, g7[7] = {0, 0, 0, 0, 0, 0, 0};
  float g15[15];
#pragma unroll
  for (int k = 0; k < 15; ++k) g15[k] = 0.f;
  const int items = B * nchunks;
  for (int it = blockIdx.y; it < items; it += nparts) {
    const int b = it / nchunks;
    const int t0 = (it % nchunks) * TC;
    const size_t base = (size_t)b * T * D + d;
    float xs[TC + HALO];  // x[t0-14 .. t0+31]
    float gs[TC + HALO];  // dS[t0 .. t0+45]
#pragma unroll
    for (int i = 0; i < TC + HALO; ++i) {
      const int tx = t0 - HALO + i;
      xs[i] = (tx >= 0 && tx < T) ? x[base + (size_t)tx * D] : 0.f;
      const int tg = t0 + i;
      gs[i] = (tg < T) ? dS[base + (size_t)tg * D] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < TC; ++i) {
      const int t = t0 + i;
      if (t >= T) break;
      // dx[t] = sum_K sum_k w_K[k] dS[t + (K-1) - k]  (dS index i + K-1-k in gs)
      float s3 = 0.f, s7 = 0.f, s15 = 0.f;
#pragma unroll
      for (int k = 0; k < 3; ++k) s3 += a3[k] * gs[i + 2 - k];
#pragma unroll
      for (int k = 0; k < 7; ++k) s7 += a7[k] * gs[i + 6 - k];
#pragma unroll
      for (int k = 0; k < 15; ++k) s15 += a15[k] * gs[i + 14 - k];
      const size_t o = base + (size_t)t * D;
      const float v = s3 + s7 + s15;
      dx[o] = accumulate ? dx[o] + v : v;
      // weight grads: x[t-(K-1)+k] * dS[t]
      const float g = gs[i];
#pragma unroll
      for (int k = 0; k < 3; ++k) g3[k] += xs[i + HALO - 2 + k] * g;
#pragma unroll
      for (int k = 0; k < 7; ++k) g7[k] += xs[i + HALO - 6 + k] * g;
#pragma unroll
      for (int k = 0; k < 15; ++k) g15[k] += xs[i + k] * g;
    }
  }
  float* pp = parts + (size_t)blockIdx.y * 25 * D + d;
#pragma unroll
  for (int k = 0; k < 3; ++k) pp[(size_t)k * D] = g3[k];
#pragma unroll
  for (int k = 0; k < 7; ++k) pp[(size_t)(3 + k) * D] = g7[k];
#pragma unroll
  for (int k = 0; k < 15; ++k) pp[(size_t)(10 + k) * D] = g15[k];
}

__global__ void conv_wgrad_reduce(const float* __restrict__ parts, int nparts, int D,
                                  float* __restrict__ dw3, float* __restrict__ dw7,
                                  float* __restrict__ dw15) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over 25*D
  if (i >= 25 * D) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += parts[(size_t)p * 25 * D + i];
  const int j = i / D, d = i % D;
  if (j < 3) dw3[j * D + d] += s;
  else if (j < 10) dw7[(j - 3) * D + d] += s;
  else dw15[(j - 10) * D + d] += s;
}

int nparts_for(int B, int T, int D) {
  const int nchunks = (T + TC - 1) / TC;
  const int groups = (D + CPB - 1) / CPB;
  int p = (148 * 6) / groups;
  if (p > MAX_PARTS) p = MAX_PARTS;
  if (p > B * nchunks) p = B * nchunks;
  return p < 1 ? 1 : p;
}

}  // namespace

cudaError_t conv_fwd(const float* x, const float* w3, const float* w7, const float* w15, float* S,
                     float* Sq, float* c7, float* c15, int B, int T, int D, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  const int nchunks = (T + TC - 1) / TC;
  dim3 grid((D + CPB - 1) / CPB, B * nchunks);
  conv_fwd_kernel<<<grid, CPB, 0, s>>>(x, w3, w7, w15, S, Sq, c7, c15, T, D, nchunks);
  return launched();
}

size_t conv_bwd_partials_floats(int B, int T, int D) {
  return (size_t)nparts_for(B, T, D) * 25 * D;
}

cudaError_t conv_bwd(const float* dS, const float* x, const float* w3, const float* w7,
                     const float* w15, float* dx, float* dw3, float* dw7, float* dw15,
                     float* partials, int B, int T, int D, int accumulate, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  const int nchunks = (T + TC - 1) / TC;
  const int np = nparts_for(B, T, D);
  dim3 grid((D + CPB - 1) / CPB, np);
  conv_bwd_kernel<<<grid, CPB, 0, s>>>(dS, x, w3, w7, w15, dx, partials, B, T, D, nchunks, np,
                                       accumulate);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  conv_wgrad_reduce<<<(25 * D + 255) / 256, 256, 0, s>>>(partials, np, D, dw3, dw7, dw15);
  return launched(2);
}

}  // namespace rnet_k
