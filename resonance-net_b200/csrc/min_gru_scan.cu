// MinGRU linear-recurrence scan, chunked and parallel over time, fused with
// the gate (z = sigmoid(pz + bz), h~ = ph + bh) and with the residual add.
//
// Reference: src/min_gru.cu:20-48 (one thread per (b,d) walking all T steps
// sequentially) and :87-126 (reverse scan + single-block bias reduction).
//
// Layout: one CTA = 8 warps = one sequence b x 32 channels; lane = channel,
// warp w = time chunk [32w, 32w+32) of the current 256-step segment.
//   pass 1: each warp composes its chunk into an affine map h -> A*h + H
//   exchange (shared memory): carry-in of chunk w = maps of chunks < w
//   pass 2: each warp re-runs its chunk from the exact carry-in with the
//           reference's own update h = (1-z) h + z h~ and writes outputs.
// Segments of 256 steps are chained through a carry so any T works.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {

namespace {

constexpr int W = 8;    // warps per CTA = chunks per segment
constexpr int CL = 32;  // steps per chunk
constexpr int SEG = W * CL;

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

__global__ void __launch_bounds__(W * 32)
    scan_fwd_kernel(const float* __restrict__ pz, const float* __restrict__ ph, int ldp,
                    const float* __restrict__ bz, const float* __restrict__ bh,
                    float* __restrict__ zo, float* __restrict__ ho, float* __restrict__ yo,
                    const float* __restrict__ res, float* __restrict__ out, int T, int D) {
  __shared__ float sA[W][32], sH[W][32];
  __shared__ float carry[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (D + 31) / 32;
  const int b = blockIdx.x / groups;
  const int d = (blockIdx.x % groups) * 32 + lane;
  const bool act = d < D;
  const float bzd = act ? bz[d] : 0.f, bhd = act ? bh[d] : 0.f;
  if (warp == 0) carry[lane] = 0.f;
  __syncthreads();
  for (int seg0 = 0; seg0 < T; seg0 += SEG) {
    const int t0 = seg0 + warp * CL;
    float z[CL], ht[CL];
    float A = 1.f, H = 0.f;
#pragma unroll
    for (int i = 0; i < CL; ++i) {
      const int t = t0 + i;
      if (act && t < T) {
        const size_t rp = ((size_t)b * T + t) * ldp + d;
        z[i] = sigmoidf_(pz[rp] + bzd);
        ht[i] = ph[rp] + bhd;
      } else {
        z[i] = 0.f;  // identity step: h unchanged
        ht[i] = 0.f;
      }
      const float a = 1.f - z[i];
      H = a * H + z[i] * ht[i];
      A = a * A;
    }
    sA[warp][lane] = A;
    sH[warp][lane] = H;
    __syncthreads();
    float h = carry[lane];
    for (int j = 0; j < warp; ++j) h = sA[j][lane] * h + sH[j][lane];
#pragma unroll
    for (int i = 0; i < CL; ++i) {
      const int t = t0 + i;
      h = (1.f - z[i]) * h + z[i] * ht[i];
      if (act && t < T) {
        const size_t o = ((size_t)b * T + t) * D + d;
        zo[o] = z[i];
        ho[o] = h;
        if (yo) yo[o] = h;
        if (out) out[o] = res[o] + h;
      }
    }
    __syncthreads();
    if (warp == W - 1) carry[lane] = h;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(W * 32)
    scan_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ z,
                    const float* __restrict__ h, const float* __restrict__ ph, int ldp,
                    const float* __restrict__ bh, float* __restrict__ dz,
                    float* __restrict__ dht, int ldd, float* __restrict__ dbz,
                    float* __restrict__ dbh, int T, int D) {
  __shared__ float sA[W][32], sH[W][32];
  __shared__ float carry[32];
  __shared__ float sbz[W][32], sbh[W][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (D + 31) / 32;
  const int b = blockIdx.x / groups;
  const int d = (blockIdx.x % groups) * 32 + lane;
  const bool act = d < D;
  const float bhd = act ? bh[d] : 0.f;
  if (warp == 0) carry[lane] = 0.f;
  float accz = 0.f, acch = 0.f;
  __syncthreads();
  const int nseg = (T + SEG - 1) / SEG;
  for (int sg = nseg - 1; sg >= 0; --sg) {
    // chunk of this warp in reverse order: warp 0 owns the LAST chunk
    const int t0 = sg * SEG + (W - 1 - warp) * CL;
    float zz[CL], g[CL];
    float A = 1.f, H = 0.f;  // dh_out = A * dh_in + H  (dh after the *= (1-z) step)
#pragma unroll
    for (int i = CL - 1; i >= 0; --i) {
      const int t = t0 + i;
      if (act && t < T) {
        const size_t o = ((size_t)b * T + t) * D + d;
        zz[i] = z[o];
        g[i] = dy[o];
      } else {
        zz[i] = 0.f;  // a = 1, no gradient injection
        g[i] = 0.f;
      }
      const float a = 1.f - zz[i];
      H = a * (H + g[i]);
      A = a * A;
    }
    sA[warp][lane] = A;
    sH[warp][lane] = H;
    __syncthreads();
    float dh = carry[lane];
    for (int j = 0; j < warp; ++j) dh = sA[j][lane] * dh + sH[j][lane];
#pragma unroll
    for (int i = CL - 1; i >= 0; --i) {
      const int t = t0 + i;
      dh += g[i];
      if (act && t < T) {
        const size_t o = ((size_t)b * T + t) * D + d;
        const size_t rp = ((size_t)b * T + t) * ldp + d;
        const size_t od = ((size_t)b * T + t) * ldd + d;
        const float htv = ph[rp] + bhd;
        const float hp = t > 0 ? h[o - D] : 0.f;
        const float zv = zz[i];
        const float vz = dh * (htv - hp) * zv * (1.f - zv);
        const float vh = dh * zv;
        dz[od] = vz;
        dht[od] = vh;
        accz += vz;
        acch += vh;
      }
      dh = dh * (1.f - zz[i]);
    }
    __syncthreads();
    if (warp == W - 1) carry[lane] = dh;
    __syncthreads();
  }
  sbz[warp][lane] = accz;
  sbh[warp][lane] = acch;
  __syncthreads();
  if (warp == 0 && act) {
    float a = 0.f, c = 0.f;
    for (int j = 0; j < W; ++j) { a += sbz[j][lane]; c += sbh[j][lane]; }
    atomicAdd(&dbz[d], a);
    atomicAdd(&dbh[d], c);
  }
}

}  // namespace

cudaError_t gru_scan_fwd(const float* pz, const float* ph, int ldp, const float* bz,
                         const float* bh, float* z, float* h, float* y, const float* res,
                         float* out, int B, int T, int D, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  const int grid = B * ((D + 31) / 32);
  scan_fwd_kernel<<<grid, W * 32, 0, s>>>(pz, ph, ldp, bz, bh, z, h, y, res, out, T, D);
  return launched();
}

cudaError_t gru_scan_bwd(const float* dy, const float* z, const float* h, const float* ph,
                         int ldp, const float* bh, float* dz, float* dht, int ldd, float* dbz,
                         float* dbh, int B, int T, int D, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  const int grid = B * ((D + 31) / 32);
  scan_bwd_kernel<<<grid, W * 32, 0, s>>>(dy, z, h, ph, ldp, bh, dz, dht, ldd, dbz, dbh, T, D);
  return launched();
}

}  // namespace rnet_k
