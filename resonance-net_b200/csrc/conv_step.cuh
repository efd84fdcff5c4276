// One causal-convolution decode step (scales 3, 7 and 15, depthwise) for four
// adjacent channels of one stream, shared by the standalone decode kernel and
// the split-K sum that also normalises the row (the step then costs no launch).
//
// ring: that stream's last 14 conv inputs, [14][D], input t at row t % 14;
// pos: index of the current token. Positions before the start contribute
// zero. The result is S = c3 + c7 + c15 with each scale summed over its taps
// in ascending order (tap k of scale K reads x[pos - (K-1) + k]), the training
// kernel's order; the current input then replaces row pos % 14.
#pragma once
#include <cuda_runtime.h>

namespace rnet_dev {

constexpr int CONV_RING = 14;

__device__ __forceinline__ float4 conv_step4(float4 x, float* ring_row, int pos,
                                             const float* __restrict__ w3,
                                             const float* __restrict__ w7,
                                             const float* __restrict__ w15, int d, int D) {
  // win[o] = x[pos - o], o = 0..14
  float4 win[CONV_RING + 1];
  win[0] = x;
#pragma unroll
  for (int o = 1; o <= CONV_RING; ++o) {
    const int t = pos - o;
    win[o] = t >= 0 ? *reinterpret_cast<const float4*>(ring_row + (size_t)(t % CONV_RING) * D + d)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float4 s3 = make_float4(0.f, 0.f, 0.f, 0.f), s7 = s3, s15 = s3;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float4 w = *reinterpret_cast<const float4*>(w3 + k * D + d);
    const float4 v = win[2 - k];
    s3.x += v.x * w.x; s3.y += v.y * w.y; s3.z += v.z * w.z; s3.w += v.w * w.w;
  }
#pragma unroll
  for (int k = 0; k < 7; ++k) {
    const float4 w = *reinterpret_cast<const float4*>(w7 + k * D + d);
    const float4 v = win[6 - k];
    s7.x += v.x * w.x; s7.y += v.y * w.y; s7.z += v.z * w.z; s7.w += v.w * w.w;
  }
#pragma unroll
  for (int k = 0; k < 15; ++k) {
    const float4 w = *reinterpret_cast<const float4*>(w15 + k * D + d);
    const float4 v = win[14 - k];
    s15.x += v.x * w.x; s15.y += v.y * w.y; s15.z += v.z * w.z; s15.w += v.w * w.w;
  }
  *reinterpret_cast<float4*>(ring_row + (size_t)(pos % CONV_RING) * D + d) = x;
  return make_float4(s3.x + s7.x + s15.x, s3.y + s7.y + s15.y, s3.z + s7.z + s15.z,
                     s3.w + s7.w + s15.w);
}

}  // namespace rnet_dev
