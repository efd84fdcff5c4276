// Slot-memory helpers around the fused score/top-2 GEMM epilogue:
// value gather, sparse backward, layout transposes, generic top-k.
//
// Reference: src/slot_memory.cu:14-77 (thread-0 top-k, stride-S value gather),
// :122-169 (backward into a dense [N,S] d_scores, global atomics on V).
// Values and keys are read from transposed shadows VT/KT [S,D] so every
// gathered slot is one contiguous row; gradients are scattered into [S,D]
// shadows with vector atomics and transposed back once per step.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

// out[j*R + i] (+)= in[i*C + j]; blockIdx.z selects matrix z of a batch:
// in + (z / 2) * in_stride2 + (z % 2) * in_stride1 -> (z % 2 ? out1 : out0) +
// (z / 2) * out_stride (keys / values of consecutive layers).
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out0,
                                 float* __restrict__ out1, size_t in_stride1, size_t in_stride2,
                                 size_t out_stride, int R, int C, int acc) {
  rnet_dev::pdl_trigger();
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int z = blockIdx.z;
  in += (size_t)(z >> 1) * in_stride2 + (size_t)(z & 1) * in_stride1;
  float* out = ((z & 1) ? out1 : out0) + (size_t)(z >> 1) * out_stride;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = in[(size_t)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) {
      float* o = out + (size_t)c * R + r;
      *o = acc ? *o + tile[threadIdx.x][i] : tile[threadIdx.x][i];
    }
  }
}

// One warp per token; lane covers 4 consecutive features per 128-wide step.
__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// r16 / dq16 (optional): bf16 outputs; the fp32 one is skipped when null.
__global__ void gather_kernel(const int* __restrict__ idx, const float* __restrict__ w,
                              const float* __restrict__ VT, float* __restrict__ r, int N, int D,
                              int S, int k, unsigned* err, __nv_bfloat16* __restrict__ r16) {
  rnet_dev::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  int id[8];
  float ww[8];
  for (int j = 0; j < k; ++j) {
    int s = idx[(size_t)warp * k + j];
    if (s < 0 || s >= S) {
      if (err && lane == 0) atomicOr(err, ERR_BAD_INDEX);
      s = 0;
    }
    id[j] = s;
    ww[j] = w[(size_t)warp * k + j];
  }
  for (int c = lane * 4; c < D; c += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(VT + (size_t)id[j] * D + c);
      acc.x += ww[j] * v.x; acc.y += ww[j] * v.y; acc.z += ww[j] * v.z; acc.w += ww[j] * v.w;
    }
    if (r) *reinterpret_cast<float4*>(r + (size_t)warp * D + c) = acc;
    if (r16) st_bf16x4(r16 + (size_t)warp * D + c, acc);
  }
}

__global__ void sparse_bwd_kernel(const float* __restrict__ dr, const int* __restrict__ idx,
                                  const float* __restrict__ w, const float* __restrict__ VT,
                                  const float* __restrict__ KT, const float* __restrict__ q,
                                  float* __restrict__ dq, float* __restrict__ dVT,
                                  float* __restrict__ dKT, int N, int D, int S, int k,
                                  unsigned* err, __nv_bfloat16* __restrict__ dq16) {
  rnet_dev::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  int id[8];
  float ww[8], dwj[8];
  for (int j = 0; j < k; ++j) {
    int s = idx[(size_t)warp * k + j];
    if (s < 0 || s >= S) {
      if (err && lane == 0) atomicOr(err, ERR_BAD_INDEX);
      s = 0;
    }
    id[j] = s;
    ww[j] = w[(size_t)warp * k + j];
    dwj[j] = 0.f;
  }
  const float* drow = dr + (size_t)warp * D;
  // dw_j = <dr, V[:, idx_j]>
  for (int c = lane * 4; c < D; c += 128) {
    const float4 g = *reinterpret_cast<const float4*>(drow + c);
    for (int j = 0; j < k; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(VT + (size_t)id[j] * D + c);
      dwj[j] += g.x * v.x + g.y * v.y + g.z * v.z + g.w * v.w;
    }
  }
  float dot = 0.f;
  for (int j = 0; j < k; ++j) {
    dwj[j] = warp_sum(dwj[j]);
    dot += ww[j] * dwj[j];
  }
  float dsc[8];
  for (int j = 0; j < k; ++j) dsc[j] = ww[j] * (dwj[j] - dot);
  const float* qrow = q + (size_t)warp * D;
  for (int c = lane * 4; c < D; c += 128) {
    const float4 g = *reinterpret_cast<const float4*>(drow + c);
    const float4 qq = *reinterpret_cast<const float4*>(qrow + c);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const float4 kv = *reinterpret_cast<const float4*>(KT + (size_t)id[j] * D + c);
      acc.x += dsc[j] * kv.x; acc.y += dsc[j] * kv.y; acc.z += dsc[j] * kv.z; acc.w += dsc[j] * kv.w;
      red_add_v4(dVT + (size_t)id[j] * D + c, ww[j] * g.x, ww[j] * g.y, ww[j] * g.z, ww[j] * g.w);
      red_add_v4(dKT + (size_t)id[j] * D + c, dsc[j] * qq.x, dsc[j] * qq.y, dsc[j] * qq.z,
                 dsc[j] * qq.w);
    }
    if (dq) *reinterpret_cast<float4*>(dq + (size_t)warp * D + c) = acc;
    if (dq16) st_bf16x4(dq16 + (size_t)warp * D + c, acc);
  }
}

// Generic top-k (k <= 8) over a materialised score matrix with the reference's
// sequential selection rule (src/slot_memory.cu:32-51), one thread per row.
// Only the per-op API uses it (k != 2); the model path selects the top-2
// inside the score GEMM epilogue and never materialises the scores.
__global__ void topk_kernel(const float* __restrict__ scores, int* __restrict__ idx,
                            float* __restrict__ w, int N, int S, int k) {
  rnet_dev::pdl_trigger();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= N) return;
  const float* sr = scores + (size_t)row * S;
  float val[8];
  int id[8];
  for (int j = 0; j < k; ++j) { val[j] = -1e30f; id[j] = 0; }
  for (int i = 0; i < S; ++i) {
    const float v = sr[i];
    int mk = 0;
    for (int j = 1; j < k; ++j)
      if (val[j] < val[mk]) mk = j;
    if (v > val[mk]) { val[mk] = v; id[mk] = i; }
  }
  float mx = val[0];
  for (int j = 1; j < k; ++j) mx = fmaxf(mx, val[j]);
  float sum = 0.f;
  for (int j = 0; j < k; ++j) { val[j] = __expf(val[j] - mx); sum += val[j]; }
  for (int j = 0; j < k; ++j) {
    idx[(size_t)row * k + j] = id[j];
    w[(size_t)row * k + j] = val[j] / sum;
  }
}

}  // namespace

cudaError_t transpose(const float* in, float* out, int R, int C, int acc, cudaStream_t s) {
  if (R <= 0 || C <= 0) return cudaSuccess;
  dim3 grid((C + 31) / 32, (R + 31) / 32, 1);
  transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(in, out, out, 0, 0, 0, R, C, acc);
  return launched();
}

cudaError_t transpose_pairs(const float* in, size_t in_stride1, size_t in_stride2, float* out0,
                            float* out1, size_t out_stride, int pairs, int R, int C, int acc,
                            cudaStream_t s) {
  if (R <= 0 || C <= 0 || pairs <= 0) return cudaSuccess;
  dim3 grid((C + 31) / 32, (R + 31) / 32, 2 * pairs);
  transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(in, out0, out1, in_stride1, in_stride2,
                                                 out_stride, R, C, acc);
  return launched();
}

cudaError_t slot_gather(const int* idx, const float* w, const float* VT, float* r, int N, int D,
                        int S, int k, unsigned* err, cudaStream_t s, __nv_bfloat16* r16) {
  if (N <= 0) return cudaSuccess;
  if (k < 1 || k > 8 || D % 4) return cudaErrorInvalidValue;
  gather_kernel<<<(N * 32 + 255) / 256, 256, 0, s>>>(idx, w, VT, r, N, D, S, k, err, r16);
  return launched();
}

cudaError_t slot_sparse_bwd(const float* dr, const int* idx, const float* w, const float* VT,
                            const float* KT, const float* q, float* dq, float* dVT, float* dKT,
                            int N, int D, int S, int k, unsigned* err, cudaStream_t s,
                            __nv_bfloat16* dq16) {
  if (N <= 0) return cudaSuccess;
  if (k < 1 || k > 8 || D % 4) return cudaErrorInvalidValue;
  sparse_bwd_kernel<<<(N * 32 + 255) / 256, 256, 0, s>>>(dr, idx, w, VT, KT, q, dq, dVT, dKT, N,
                                                         D, S, k, err, dq16);
  return launched();
}

cudaError_t topk_rows(const float* scores, int* idx, float* w, int N, int S, int k,
                      cudaStream_t s) {
  if (N <= 0) return cudaSuccess;
  if (k < 1 || k > 8) return cudaErrorInvalidValue;
  topk_kernel<<<(N + 127) / 128, 128, 0, s>>>(scores, idx, w, N, S, k);
  return launched();
}

}  // namespace rnet_k
