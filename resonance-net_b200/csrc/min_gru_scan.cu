// MinGRU linear-recurrence scan, chunked and parallel over time, fused with
// the gate (z = sigmoid(pz + bz), h~ = ph + bh) and with the residual add.
//
// Reference: src/min_gru.cu:20-48 (one thread per (b,d) walking all T steps
// sequentially) and :87-126 (reverse scan + single-block bias reduction).
//
// Layout: one CTA = 8 warps = one sequence b x 32 channels; lane = channel,
// warp w = time chunk [32w, 32w+32) of the current 256-step segment.
//   stage:  the segment's inputs ([256 steps x 32 channels] tiles) are copied
//           global -> shared with cp.async (16 B per copy, all in flight at
//           once), so the serial part of the scan never waits on DRAM
//   pass 1: each warp composes its chunk into an affine map h -> A*h + H
//   carry:  chunk w's carry-in = the maps of chunks < w (shared memory)
//   pass 2: each warp re-runs its chunk from the exact carry-in with the
//           reference's own update h = (1-z) h + z h~ and writes outputs.
// Segments of 256 steps are chained through a carry so any T works.
#include "common.cuh"
#include "kernels.cuh"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int W = 8;    // warps per CTA = chunks per segment
constexpr int CL = 32;  // steps per chunk
constexpr int SEG = W * CL;
constexpr int CW = 32;  // channels per CTA
constexpr int TILE = SEG * CW;  // floats per staged tile


__device__ __forceinline__ void cp_async16(float* smem, const float* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Stage rows [seg0, seg0+SEG) x channels [c0, c0+32) of a row-major [B*T, ld]
// array into a [SEG][CW] tile (zero-filled outside T / D).
__device__ __forceinline__ void stage(float* tile, const float* src, int ld, int b, int T, int D,
                                      int seg0, int c0) {
  for (int q = threadIdx.x; q < SEG * 8; q += W * 32) {
    const int row = q >> 3, part = q & 7;
    const int t = seg0 + row, ch = c0 + part * 4;
    const bool valid = t < T && ch < D;
    const float* g = valid ? src + ((size_t)b * T + t) * ld + ch : src;
    cp_async16(tile + row * CW + part * 4, g, valid);
  }
}

// Output set of the forward scan (compile-time, so the step loops carry no
// per-step tests): DIFF: `ho` receives e = h~ - h_prev instead of h; Y: y = h;
// OUT: out = res + h; OUT2: a second copy of out.
enum : int { F_DIFF = 1, F_Y = 2, F_OUT = 4, F_OUT2 = 8 };

// Pass 2 of one warp's chunk: re-run the chunk from its exact carry-in and
// write the outputs. FULL: every step of the chunk is inside [0, T).
template <int FL, bool FULL>
__device__ __forceinline__ float scan_fwd_emit(const float* sZ, const float* sT, const float* sR,
                                               int r0, int lane, float h, int n, size_t o0, int D,
                                               float* zo, float* ho, float* yo, float* out,
                                               float* out2) {
  size_t o = o0;
#pragma unroll 8
  for (int i = 0; i < CL; ++i) {
    if (!FULL && i >= n) break;
    const int row = r0 + i;
    const float z = sZ[row * CW + lane];
    const float ht = sT[row * CW + lane];
    const float hp = h;
    h = (1.f - z) * h + z * ht;
    zo[o] = z;
    ho[o] = (FL & F_DIFF) ? ht - hp : h;
    if (FL & F_Y) yo[o] = h;
    if (FL & F_OUT) {
      const float r = sR[row * CW + lane] + h;
      out[o] = r;
      if (FL & F_OUT2) out2[o] = r;
    }
    o += D;
  }
  return h;
}

template <int FL>
__global__ void __launch_bounds__(W * 32)
    scan_fwd_kernel(const float* __restrict__ pz, const float* __restrict__ ph, int ldp,
                    const float* __restrict__ bz, const float* __restrict__ bh,
                    float* __restrict__ zo, float* __restrict__ ho, float* __restrict__ yo,
                    const float* __restrict__ res, float* __restrict__ out,
                    float* __restrict__ out2, int T, int D) {
  rnet_dev::pdl_trigger();
  extern __shared__ float smem[];
  float* sZ = smem;             // pz, then z
  float* sT = smem + TILE;      // ph, then h~
  float* sR = smem + 2 * TILE;  // residual input (OUT only)
  __shared__ float sA[W][32], sH[W][32];
  __shared__ float carry[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (D + CW - 1) / CW;
  const int b = blockIdx.x / groups;
  const int c0 = (blockIdx.x % groups) * CW;
  const int d = c0 + lane;
  const bool act = d < D;
  const float bzd = act ? bz[d] : 0.f, bhd = act ? bh[d] : 0.f;
  if (warp == 0) carry[lane] = 0.f;
  for (int seg0 = 0; seg0 < T; seg0 += SEG) {
    stage(sZ, pz, ldp, b, T, D, seg0, c0);
    stage(sT, ph, ldp, b, T, D, seg0, c0);
    if (FL & F_OUT) stage(sR, res, D, b, T, D, seg0, c0);
    cp_async_wait_all();
    __syncthreads();
    const int r0 = warp * CL;
    const int n = T - (seg0 + r0) < CL ? T - (seg0 + r0) : CL;  // live steps of the chunk
    float A = 1.f, H = 0.f;
#pragma unroll 8
    for (int i = 0; i < CL; ++i) {
      const int row = r0 + i;
      const bool live = act && i < n;
      // steps past T (and lanes past D) are identity steps (z = 0: h unchanged);
      // z = 1 / (1 + exp(-(pz + bz))) with the fast divide (a few ulp)
      const float z = live ? sigmoid_fast(sZ[row * CW + lane] + bzd) : 0.f;
      const float ht = live ? sT[row * CW + lane] + bhd : 0.f;
      sZ[row * CW + lane] = z;
      sT[row * CW + lane] = ht;
      const float a = 1.f - z;
      H = a * H + z * ht;
      A = a * A;
    }
    sA[warp][lane] = A;
    sH[warp][lane] = H;
    __syncthreads();
    float h = carry[lane];
    for (int j = 0; j < warp; ++j) h = sA[j][lane] * h + sH[j][lane];
    if (act && n > 0) {
      const size_t o0 = ((size_t)b * T + seg0 + r0) * D + d;
      if (n == CL)
        h = scan_fwd_emit<FL, true>(sZ, sT, sR, r0, lane, h, n, o0, D, zo, ho, yo, out, out2);
      else
        h = scan_fwd_emit<FL, false>(sZ, sT, sR, r0, lane, h, n, o0, D, zo, ho, yo, out, out2);
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
                    float* __restrict__ dbh, int T, int D, __nv_bfloat16* __restrict__ dz16,
                    __nv_bfloat16* __restrict__ dht16) {
  rnet_dev::pdl_trigger();
  extern __shared__ float smem[];
  float* sZ = smem;
  float* sG = smem + TILE;
  float* sP = smem + 2 * TILE;
  __shared__ float sA[W][32], sH[W][32];
  __shared__ float carry[32];
  __shared__ float sbz[W][32], sbh[W][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (D + CW - 1) / CW;
  const int b = blockIdx.x / groups;
  const int c0 = (blockIdx.x % groups) * CW;
  const int d = c0 + lane;
  const bool act = d < D;
  const float bhd = act && ph ? bh[d] : 0.f;
  if (warp == 0) carry[lane] = 0.f;
  float accz = 0.f, acch = 0.f;
  const int nseg = (T + SEG - 1) / SEG;
  for (int sg = nseg - 1; sg >= 0; --sg) {
    const int seg0 = sg * SEG;
    stage(sZ, z, D, b, T, D, seg0, c0);
    stage(sG, dy, D, b, T, D, seg0, c0);
    if (ph) stage(sP, ph, ldp, b, T, D, seg0, c0);
    else stage(sP, h, D, b, T, D, seg0, c0);  // h holds e = h~ - h_prev
    cp_async_wait_all();
    __syncthreads();
    // warp 0 owns the LAST chunk of the segment (reverse time order)
    const int r0 = (W - 1 - warp) * CL;
    float A = 1.f, H = 0.f;  // dh_out = A * dh_in + H  (dh after the *= (1-z) step)
#pragma unroll 8
    for (int i = CL - 1; i >= 0; --i) {
      const int row = r0 + i;
      const float a = 1.f - sZ[row * CW + lane];  // zero-filled past T: a = 1, g = 0
      H = a * (H + sG[row * CW + lane]);
      A = a * A;
    }
    sA[warp][lane] = A;
    sH[warp][lane] = H;
    __syncthreads();
    float dh = carry[lane];
    for (int j = 0; j < warp; ++j) dh = sA[j][lane] * dh + sH[j][lane];
#pragma unroll 8
    for (int i = CL - 1; i >= 0; --i) {
      const int row = r0 + i;
      const int t = seg0 + row;
      const float zv = sZ[row * CW + lane];
      dh += sG[row * CW + lane];
      if (act && t < T) {
        const size_t o = ((size_t)b * T + t) * D + d;
        const size_t od = ((size_t)b * T + t) * ldd + d;
        float e;
        if (ph) {
          const float htv = sP[row * CW + lane] + bhd;
          const float hp = t > 0 ? h[o - D] : 0.f;
          e = htv - hp;
        } else {
          e = sP[row * CW + lane];
        }
        const float vz = dh * e * zv * (1.f - zv);
        const float vh = dh * zv;
        if (dz16) {
          dz16[od] = __float2bfloat16_rn(vz);
          dht16[od] = __float2bfloat16_rn(vh);
        } else {
          dz[od] = vz;
          dht[od] = vh;
        }
        accz += vz;
        acch += vh;
      }
      dh = dh * (1.f - zv);
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

template <class K>
void allow_smem(K kernel, size_t bytes) {
  static bool done = false;
  if (!done) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    done = true;
  }
}

}  // namespace

template <int FL>
void launch_fwd(int grid, size_t smem, cudaStream_t s, const float* pz, const float* ph, int ldp,
                const float* bz, const float* bh, float* z, float* h, float* y, const float* res,
                float* out, float* out2, int T, int D) {
  static bool done = false;
  if (!done) {
    cudaFuncSetAttribute(scan_fwd_kernel<FL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(3 * TILE * sizeof(float)));
    done = true;
  }
  scan_fwd_kernel<FL><<<grid, W * 32, smem, s>>>(pz, ph, ldp, bz, bh, z, h, y, res, out, out2, T,
                                                 D);
}

cudaError_t gru_scan_fwd(const float* pz, const float* ph, int ldp, const float* bz,
                         const float* bh, float* z, float* h, float* y, const float* res,
                         float* out, int B, int T, int D, cudaStream_t s, bool h_as_diff,
                         float* out2) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 4 || ldp % 4) return cudaErrorInvalidValue;
  if (out2 && !out) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(out ? 3 : 2) * TILE * sizeof(float);
  const int grid = B * ((D + CW - 1) / CW);
  const int fl = (h_as_diff ? F_DIFF : 0) | (y ? F_Y : 0) | (out ? F_OUT : 0) | (out2 ? F_OUT2 : 0);
#define RNET_SCAN_CASE(F)                                                                 \
  case F:                                                                                 \
    launch_fwd<F>(grid, smem, s, pz, ph, ldp, bz, bh, z, h, y, res, out, out2, T, D);     \
    break;
  switch (fl) {
    RNET_SCAN_CASE(0) RNET_SCAN_CASE(1) RNET_SCAN_CASE(2) RNET_SCAN_CASE(3)
    RNET_SCAN_CASE(4) RNET_SCAN_CASE(5) RNET_SCAN_CASE(6) RNET_SCAN_CASE(7)
    RNET_SCAN_CASE(12) RNET_SCAN_CASE(13) RNET_SCAN_CASE(14) RNET_SCAN_CASE(15)
    default: return cudaErrorInvalidValue;
  }
#undef RNET_SCAN_CASE
  return launched();
}

cudaError_t gru_scan_bwd(const float* dy, const float* z, const float* h, const float* ph,
                         int ldp, const float* bh, float* dz, float* dht, int ldd, float* dbz,
                         float* dbh, int B, int T, int D, cudaStream_t s, __nv_bfloat16* dzh16) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 4 || ldp % 4) return cudaErrorInvalidValue;
  const size_t smem = (size_t)3 * TILE * sizeof(float);
  allow_smem(scan_bwd_kernel, smem);
  const int grid = B * ((D + CW - 1) / CW);
  __nv_bfloat16* dht16 = dzh16 ? dzh16 + (dht - dz) : nullptr;
  scan_bwd_kernel<<<grid, W * 32, smem, s>>>(dy, z, h, ph, ldp, bh, dz, dht, ldd, dbz, dbh, T, D,
                                             dzh16, dht16);
  return launched();
}

}  // namespace rnet_k
