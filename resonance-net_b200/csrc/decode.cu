// Kernels of the recurrent (O(1)-state) decode path.
//
// The reference has no decode path: its `infer` re-runs the whole prefix for
// every token at batch 1 (src/main.cpp:316-325) and `generate()` is declared
// but never defined (include/resonance_net.h:82-83). The state that makes a
// single-token step exact is, per layer and stream: the last 14 inputs of the
// causal convolutions (a ring indexed by position mod 14) and the MinGRU h.
#include "common.cuh"
#include "conv_step.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int RING = rnet_dev::CONV_RING;

// S = c3 + c7 + c15 of the current input row n[m] and the ring of the 14
// previous rows (conv_step4); then the current row is written into the ring
// at pos % 14. Positions before the start of the sequence contribute zero
// (the ring is zero-initialised / filled by prefill). A thread per 4 channels.
__global__ void decode_conv_kernel(const float* __restrict__ n, float* __restrict__ ring,
                                   const int* __restrict__ pos_ptr, const float* __restrict__ w3,
                                   const float* __restrict__ w7, const float* __restrict__ w15,
                                   float* __restrict__ S, int M, int D) {
  rnet_dev::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int D4 = D >> 2;
  if (i >= M * D4) return;
  const int m = i / D4, d = (i % D4) * 4;
  const float4 x = *reinterpret_cast<const float4*>(n + (size_t)m * D + d);
  *reinterpret_cast<float4*>(S + (size_t)m * D + d) =
      rnet_dev::conv_step4(x, ring + (size_t)m * RING * D, *pos_ptr, w3, w7, w15, d, D);
}

// After a prefill of T steps: h_state[m] = h[m, T-1]; ring[t % 14] = n1[m, t]
// for t in [T-14, T-1] (zero for t < 0).
__global__ void extract_state_kernel(const float* __restrict__ n1, const float* __restrict__ h,
                                     float* __restrict__ ring, float* __restrict__ hs, int M,
                                     int T, int D) {
  rnet_dev::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * D) return;
  const int m = i / D, d = i % D;
  hs[i] = h[((size_t)m * T + T - 1) * D + d];
  float* rg = ring + (size_t)m * RING * D + d;
  for (int j = 0; j < RING; ++j) {
    const int t = T - RING + j;
    if (t >= 0) rg[(size_t)(t % RING) * D] = n1[((size_t)m * T + t) * D + d];
    else rg[(size_t)(((t % RING) + RING) % RING) * D] = 0.f;
  }
}

// Row gather: out[m] = x[m*T + T-1]
__global__ void last_rows_kernel(const float* __restrict__ x, float* __restrict__ out, int M,
                                 int T, int D) {
  rnet_dev::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * D) return;
  const int m = i / D, d = i % D;
  out[i] = x[((size_t)m * T + T - 1) * D + d];
}

// Greedy argmax per row (first maximum wins), one warp per row; writes the
// token to tok[m], to out[m] (if given) and advances the device position once.
__global__ void argmax_kernel(const float* __restrict__ logits, int M, int V,
                              int* __restrict__ tok, int* __restrict__ out,
                              int* __restrict__ pos_ptr) {
  rnet_dev::pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp < M) {
    const float* l = logits + (size_t)warp * V;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < V; c += 32) {
      const float v = l[c];
      if (v > best || (v == best && c < bi)) { best = v; bi = c; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      tok[warp] = bi;
      if (out) out[warp] = bi;
    }
  }
  if (pos_ptr && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(pos_ptr, 1);
}

// Counter-based uniform in [0, 1) with 24 random bits: splitmix64 of
// (seed, stream, position). The same function is restated by the tests.
__device__ __forceinline__ float sample_uniform(unsigned long long seed, int stream, int pos) {
  unsigned long long z = seed + 0x9E3779B97F4A7C15ull * (1ull + (unsigned long long)stream) +
                         0xD1B54A32D192ED03ull * (unsigned long long)(unsigned)pos;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

// Temperature + top-p (nucleus) sampling per row, the rule of the
// reference's infer loop (src/main.cpp:327-360): p = exp((l - max) / T)
// summed in index order and normalised; probabilities sorted descending
// (ties: lower token first); cutoff = first prefix whose running sum reaches
// top_p (all V if none does); r = u * (sum of the kept probabilities); the
// token is the first in sorted order whose running sum reaches r. The sums
// run sequentially in the reference's order (thread 0). One CTA per row,
// blockDim = SORT_N >= V. u comes from sample_uniform(seed, row, position
// of the sampled token) where that position is *pos_ptr + advance;
// advance = 1 also advances *pos_ptr (decode step), 0 leaves it (prefill).
constexpr int SORT_N = 1024;
__global__ void __launch_bounds__(SORT_N) sample_topp_kernel(
    const float* __restrict__ logits, int M, int V, float temperature, float top_p,
    unsigned long long seed, int* __restrict__ tok, int* __restrict__ pos_ptr, int advance) {
  rnet_dev::pdl_trigger();
  __shared__ float p[SORT_N];
  __shared__ int id[SORT_N];
  __shared__ float red[32];
  const int row = blockIdx.x, t = threadIdx.x, n = blockDim.x;
  const float* l = logits + (size_t)row * V;
  const float v = t < V ? l[t] : -INFINITY;
  // row maximum
  float m = rnet_dev::warp_max(v);
  if ((t & 31) == 0) red[t >> 5] = m;
  __syncthreads();
  if (t < 32) {
    float x = t < (n >> 5) ? red[t] : -INFINITY;
    x = rnet_dev::warp_max(x);
    if (t == 0) red[0] = x;
  }
  __syncthreads();
  const float mx = red[0];
  p[t] = t < V ? expf((v - mx) / temperature) : -1.0f;  // padding sorts last
  id[t] = t;
  __syncthreads();
  if (t == 0) {
    float sum = 0.0f;
    for (int i = 0; i < V; ++i) sum += p[i];
    red[1] = sum;
  }
  __syncthreads();
  if (t < V) p[t] /= red[1];
  __syncthreads();
  // bitonic sort, descending by probability, ascending token on ties
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int o = t ^ j;
      if (o > t) {
        const float pa = p[t], pb = p[o];
        const int ia = id[t], ib = id[o];
        const bool a_first = pa > pb || (pa == pb && ia < ib);
        const bool desc = (t & k) == 0;
        if (desc != a_first) {
          p[t] = pb; p[o] = pa;
          id[t] = ib; id[o] = ia;
        }
      }
      __syncthreads();
    }
  }
  if (t == 0) {
    float cum = 0.0f;
    int cutoff = V;
    for (int i = 0; i < V; ++i) {
      cum += p[i];
      if (cum >= top_p) { cutoff = i + 1; break; }
    }
    float resum = 0.0f;
    for (int i = 0; i < cutoff; ++i) resum += p[i];
    const int at = *pos_ptr + advance;
    const float r = sample_uniform(seed, row, at) * resum;
    int pick = id[0];
    cum = 0.0f;
    for (int i = 0; i < cutoff; ++i) {
      cum += p[i];
      if (cum >= r) { pick = id[i]; break; }
    }
    tok[row] = pick;
  }
  // every row has read *pos_ptr before any CTA could advance it: the advance
  // happens in a separate single-thread launch (see sample_rows)
}

__global__ void advance_pos_kernel(int* pos_ptr) {
  rnet_dev::pdl_trigger();
  if (threadIdx.x == 0) atomicAdd(pos_ptr, 1);
}

// Top-2 of each score row by the reference's sequential rule (walk the slots
// in order; a score strictly above the smaller held score replaces the first
// such minimum), then softmax over the pair (src/slot_memory.cu:40-51).
// The held pair always holds the two largest scores seen so far, so slot i
// changes the state only if its score exceeds the second largest of slots
// [0, i). One warp per row, lane l owning slots [32l, 32l+32): a warp scan of
// (largest, second largest) gives every lane the values held when its chunk
// starts; each lane flags the slots that would enter; only those are then
// replayed in slot order, the held pair (with positions) passed lane to lane.
__device__ __forceinline__ void top2_merge(float& a1, float& a2, float b1, float b2) {
  // multiset top-2 of {a1, a2, b1, b2} (a1 >= a2, b1 >= b2)
  const float m1 = fmaxf(a1, b1);
  const float m2 = fmaxf(fminf(a1, b1), fmaxf(a2, b2));
  a1 = m1;
  a2 = m2;
}

// The scan itself, for one warp: ld(s) gives the score of slot s. Leaves the
// held pair (values h0, h1 at positions i0, i1) uniform across the warp.
template <class Load>
__device__ __forceinline__ void top2_scan_warp(Load ld, int S, int lane, float& h0, float& h1,
                                               int& i0, int& i1) {
  const float NEG = -1e30f;  // the reference's initial held value
  h0 = NEG;
  h1 = NEG;
  i0 = 0;
  i1 = 0;
  for (int base = 0; base < S; base += 32 * 32) {
    const int s0 = base + lane * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = s0 + j < S ? ld(s0 + j) : NEG;
    // chunk top-2 (values)
    float c1 = NEG, c2 = NEG;
#pragma unroll
    for (int j = 0; j < 32; ++j) top2_merge(c1, c2, v[j], NEG);
    // inclusive warp scan, then the values held when this lane's chunk starts
    float p1 = c1, p2 = c2;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float q1 = __shfl_up_sync(0xffffffffu, p1, o);
      const float q2 = __shfl_up_sync(0xffffffffu, p2, o);
      if (lane >= o) top2_merge(p1, p2, q1, q2);
    }
    float e1 = __shfl_up_sync(0xffffffffu, p1, 1), e2 = __shfl_up_sync(0xffffffffu, p2, 1);
    if (lane == 0) { e1 = NEG; e2 = NEG; }
    top2_merge(e1, e2, fmaxf(h0, h1), fminf(h0, h1));  // state carried from earlier blocks
    // flag the slots that enter: strictly above the running second largest
    unsigned flags = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (s0 + j < S && v[j] > e2) {
        flags |= 1u << j;
        top2_merge(e1, e2, v[j], NEG);
      }
    }
    // replay the flagged slots in order with positions, lane by lane
    unsigned busy = __ballot_sync(0xffffffffu, flags != 0);
    while (busy) {
      const int src = __ffs(busy) - 1;
      busy &= busy - 1;
      if (lane == src) {
        unsigned f = flags;
        while (f) {
          const int j = __ffs(f) - 1;
          f &= f - 1;
          const float x = v[j];
          const bool m1 = h1 < h0;
          const float hm = m1 ? h1 : h0;
          if (x > hm) {
            if (m1) { h1 = x; i1 = s0 + j; } else { h0 = x; i0 = s0 + j; }
          }
        }
      }
      h0 = __shfl_sync(0xffffffffu, h0, src);
      h1 = __shfl_sync(0xffffffffu, h1, src);
      i0 = __shfl_sync(0xffffffffu, i0, src);
      i1 = __shfl_sync(0xffffffffu, i1, src);
    }
  }
}

// The decode step's slot sublayer after the score GEMM, one 256-thread CTA
// per row:
//  1. all threads sum the score GEMM's partial planes in plane order (the
//     split-K sum's order, so the same values), float4-coalesced, into shared
//     memory padded by one word per 32 (slot s at s + s / 32, so the scan's
//     lane-strided reads are free of bank conflicts);
//  2. warp 0 runs the sequential top-2 scan and the pair softmax;
//  3. all threads add w0 VP[i0] + w1 VP[i1] (VP = V * proj_out^T, the slot
//     sublayer's output) into the residual row, then write its RMSNorm.
constexpr int SLOT_ROW_THREADS = 256;

__global__ void __launch_bounds__(SLOT_ROW_THREADS)
    slot_row_kernel(const float* __restrict__ planes, int n_planes, int* __restrict__ idx,
                    float* __restrict__ w, int M, int S, const float* __restrict__ VP,
                    float* __restrict__ x, int D, const float* __restrict__ nw,
                    float* __restrict__ ny, float eps) {
  rnet_dev::pdl_trigger();
  extern __shared__ float sc[];  // S + S / 32 floats
  __shared__ float red[SLOT_ROW_THREADS / 32];
  __shared__ float pick_w[2];
  __shared__ int pick_i[2];
  const size_t row = blockIdx.x;
  const size_t plane = (size_t)M * S;
  const float* src = planes + row * S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int q = tid; q < (S >> 2); q += SLOT_ROW_THREADS) {
    float4 a = *reinterpret_cast<const float4*>(src + 4 * q);
    for (int k0 = 1; k0 < n_planes; k0 += 8) {
      float4 b[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (k0 + j < n_planes)
          b[j] = *reinterpret_cast<const float4*>(src + (k0 + j) * plane + 4 * q);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (k0 + j < n_planes) { a.x += b[j].x; a.y += b[j].y; a.z += b[j].z; a.w += b[j].w; }
    }
    const int s0 = 4 * q, p = s0 + (s0 >> 5);  // the 4 slots share one 32-slot group
    sc[p] = a.x;
    sc[p + 1] = a.y;
    sc[p + 2] = a.z;
    sc[p + 3] = a.w;
  }
  __syncthreads();
  if (warp == 0) {
    float h0, h1;
    int i0, i1;
    top2_scan_warp([&](int j) { return sc[j + (j >> 5)]; }, S, lane, h0, h1, i0, i1);
    const float mx = fmaxf(h0, h1);
    const float e0 = __expf(h0 - mx), e1 = __expf(h1 - mx);
    const float sum = e0 + e1;
    if (lane == 0) {
      const float w0 = e0 / sum, w1 = e1 / sum;
      pick_w[0] = w0;
      pick_w[1] = w1;
      pick_i[0] = i0;
      pick_i[1] = i1;
      idx[2 * row] = i0;
      idx[2 * row + 1] = i1;
      w[2 * row] = w0;
      w[2 * row + 1] = w1;
    }
  }
  __syncthreads();
  const int id[2] = {pick_i[0], pick_i[1]};
  const float ww[2] = {pick_w[0], pick_w[1]};
  float* xr = x + row * D;
  float ss = 0.f;
  for (int c = tid * 4; c < D; c += SLOT_ROW_THREADS * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < 2; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(VP + (size_t)id[j] * D + c);
      acc.x += ww[j] * v.x; acc.y += ww[j] * v.y; acc.z += ww[j] * v.z; acc.w += ww[j] * v.w;
    }
    float4 xv = *reinterpret_cast<const float4*>(xr + c);
    xv.x += acc.x; xv.y += acc.y; xv.z += acc.z; xv.w += acc.w;
    *reinterpret_cast<float4*>(xr + c) = xv;
    ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < SLOT_ROW_THREADS / 32; ++k) t += red[k];
  const float ri = rsqrtf(t / (float)D + eps);
  float* yr = ny + row * D;
  for (int c = tid * 4; c < D; c += SLOT_ROW_THREADS * 4) {
    const float4 xv = *reinterpret_cast<const float4*>(xr + c);
    const float4 g = *reinterpret_cast<const float4*>(nw + c);
    *reinterpret_cast<float4*>(yr + c) =
        make_float4(xv.x * ri * g.x, xv.y * ri * g.y, xv.z * ri * g.z, xv.w * ri * g.w);
  }
}

// out[s, j] = sum_d A[s, d] * B[d * bd + j * bj] over d < K, accumulated in
// double (A: [R, K] rows, out: [R, J] rows). 32 x 32 output tiles, 256
// threads, 4 outputs per thread; K staged 32 at a time through shared memory.
__global__ void __launch_bounds__(256) fold_kernel(const float* __restrict__ A,
                                                   const float* __restrict__ B, size_t bd,
                                                   size_t bj, float* __restrict__ out, int R,
                                                   int J, int K) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // ty: 0..7
  const int r0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      const int rr = r0 + i, kk = k0 + tx;
      As[i][tx] = (rr < R && kk < K) ? A[(size_t)rr * K + kk] : 0.f;
      const int dd = k0 + i, jj = j0 + tx;
      Bs[i][tx] = (dd < K && jj < J) ? B[dd * bd + jj * bj] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const double b = (double)Bs[kk][tx];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] += (double)As[ty + 8 * q][kk] * b;
    }
    __syncthreads();
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int rr = r0 + ty + 8 * q, jj = j0 + tx;
    if (rr < R && jj < J) out[(size_t)rr * J + jj] = (float)acc[q];
  }
}

}  // namespace

cudaError_t topk2_gather_residual_norm(const float* planes, int n_planes, int* idx, float* w,
                                       int M, int S, const float* VP, float* x, int D,
                                       const float* nw, float* ny, float eps, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if (D % 4 || S % 4 || !VP || !x || !nw || !ny || n_planes < 1) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(S + S / 32 + 1) * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static int smem_set = 0;  // opt in above 48 KB once (largest size asked so far)
  if ((int)smem > 48 * 1024 && (int)smem > smem_set) {
    cudaError_t e = cudaFuncSetAttribute(slot_row_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    smem_set = (int)smem;
  }
  slot_row_kernel<<<M, SLOT_ROW_THREADS, smem, s>>>(planes, n_planes, idx, w, M, S, VP, x, D,
                                                    nw, ny, eps);
  return launched();
}

cudaError_t fold_rows(const float* A, const float* B, size_t bd, size_t bj, float* out, int R,
                      int J, int K, cudaStream_t s) {
  if (R <= 0 || J <= 0) return cudaSuccess;
  dim3 grid((J + 31) / 32, (R + 31) / 32);
  fold_kernel<<<grid, 256, 0, s>>>(A, B, bd, bj, out, R, J, K);
  return launched();
}

cudaError_t decode_conv(const float* n, float* ring, const int* pos, const float* w3,
                        const float* w7, const float* w15, float* S, int M, int D,
                        cudaStream_t s) {
  if (D % 4) return cudaErrorInvalidValue;
  decode_conv_kernel<<<(M * D / 4 + 255) / 256, 256, 0, s>>>(n, ring, pos, w3, w7, w15, S, M, D);
  return launched();
}

cudaError_t decode_extract_state(const float* n1, const float* h, float* ring, float* hs, int M,
                                 int T, int D, cudaStream_t s) {
  extract_state_kernel<<<(M * D + 255) / 256, 256, 0, s>>>(n1, h, ring, hs, M, T, D);
  return launched();
}

cudaError_t last_rows(const float* x, float* out, int M, int T, int D, cudaStream_t s) {
  last_rows_kernel<<<(M * D + 255) / 256, 256, 0, s>>>(x, out, M, T, D);
  return launched();
}

cudaError_t argmax_rows(const float* logits, int M, int V, int* tok, int* out, int* pos,
                        cudaStream_t s) {
  argmax_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(logits, M, V, tok, out, pos);
  return launched();
}

cudaError_t sample_rows(const float* logits, int M, int V, float temperature, float top_p,
                        unsigned long long seed, int* tok, int* pos, int advance, cudaStream_t s) {
  if (temperature <= 0.0f) return argmax_rows(logits, M, V, tok, nullptr, advance ? pos : nullptr, s);
  if (V > SORT_N) return cudaErrorInvalidValue;
  int n = 32;
  while (n < V) n <<= 1;
  sample_topp_kernel<<<M, n, 0, s>>>(logits, M, V, temperature, top_p, seed, tok, pos, advance);
  cudaError_t e = launched();
  if (e != cudaSuccess || !advance) return e;
  advance_pos_kernel<<<1, 32, 0, s>>>(pos);
  return launched();
}

}  // namespace rnet_k
