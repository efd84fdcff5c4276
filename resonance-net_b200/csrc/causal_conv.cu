// Multi-scale depthwise causal convolution (k = 3, 7, 15) fused into one pass.
//
// Reference: src/causal_conv.cu:9-30 (one depthwise kernel launched per scale),
// :33-39 + :61-71 (sum3 into the c3 slot), :85-130 and :150-187 (data and
// weight gradients, the weight gradient on only K blocks).
//
// Layout: a persistent CTA owns 32 channels (lane = channel) and walks the
// 128-step tiles of the sequences. A tile plus its 14-step halo ([142 rows x
// 32 channels]) is copied global -> shared with cp.async (16 B per copy), three
// tiles in flight per CTA; warp w runs steps [16w, 16w+16) of a tile from
// shared memory with a 30-sample register window and writes each output row
// (128 B per warp) coalesced. The weight gradient is a deterministic two-level
// reduction: warps of a CTA in fixed order, then CTA partials in fixed order.
// Taps are merged by lag (see fwd_steps_merged / conv_bwd_kernel): fp32 sums
// in a different association than the reference's per-scale sums.
//
// The C-ABI forward (which returns c7 and c15) sums per scale in the
// reference's order (sum += x*w over taps in increasing k, zero left padding;
// S = (c3 + c7) + c15 as its sum3); the model path merges taps by lag.
#include <cstdlib>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels.cuh"
#include "status.h"

namespace rnet_k {
using namespace rnet_dev;

namespace {

constexpr int HALO = 14;             // max kernel size - 1
constexpr int CW = 32;               // channels per CTA (lane = channel)
constexpr int NW = 8;                // warps per CTA
constexpr int STEPS = 16;            // steps per warp
constexpr int TS = NW * STEPS;       // steps per tile
constexpr int ROWS = TS + HALO;      // staged rows per tile
constexpr int WIN = STEPS + HALO;    // register window per warp
constexpr int MAX_PARTS = 64;        // weight-gradient partials per channel group
constexpr int PIPE = 3;              // forward: tiles in flight per CTA (cp.async groups)
constexpr int PIPE_B = 2;            // backward: {x, dS} tile pairs in flight per CTA

__device__ __forceinline__ void cp_async16(float* smem, const float* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Stage rows t = t_first .. t_first + ROWS - 1 of sequence b, channels
// [c0, c0 + 32) of a [B, T, D] array into tile[ROWS][CW]; zero outside [0, T)
// and past D.
__device__ __forceinline__ void stage(float (*tile)[CW], const float* src, int b, int T, int D,
                                      int t_first, int c0) {
  for (int q = threadIdx.x; q < ROWS * (CW / 4); q += NW * 32) {
    const int row = q / (CW / 4), part = q % (CW / 4);
    const int t = t_first + row, ch = c0 + part * 4;
    const bool valid = t >= 0 && t < T && ch < D;
    const float* g = valid ? src + ((size_t)b * T + t) * D + ch : src;
    cp_async16(&tile[row][part * 4], g, valid);
  }
}

// Outputs of one warp's STEPS steps from its register window (output step i
// uses x[t-(K-1)+k] = win[i + HALO - (K-1) + k]). WQ: also Sq = S + c7 + c15
// (the reference's dmix operand); WC: also c7, c15. FULL: all STEPS steps
// exist (no bounds test in the unrolled loop).
template <bool WQ, bool WC, bool FULL>
__device__ __forceinline__ void fwd_steps(const float (&win)[WIN], const float (&a3)[3],
                                          const float (&a7)[7], const float (&a15)[15], float* pS,
                                          float* pQ, float* p7, float* p15, int n, int D) {
#pragma unroll
  for (int i = 0; i < STEPS; ++i) {
    if (!FULL && i >= n) break;
    float s3 = 0.f, s7 = 0.f, s15 = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) s3 += win[i + HALO - 2 + k] * a3[k];
#pragma unroll
    for (int k = 0; k < 7; ++k) s7 += win[i + HALO - 6 + k] * a7[k];
#pragma unroll
    for (int k = 0; k < 15; ++k) s15 += win[i + k] * a15[k];
    const float sum = s3 + s7 + s15;
    *pS = sum;
    pS += D;
    if (WQ) {
      *pQ = sum + s7 + s15;
      pQ += D;
    }
    if (WC) {
      *p7 = s7;
      *p15 = s15;
      p7 += D;
      p15 += D;
    }
  }
}

// Model-path outputs (S, optionally Sq) with the taps merged by lag: tap k of
// kernel K reads x[t - l] with l = K-1-k, so c7 + c15 = sum_l u[l] x[t - l],
// u[l] = w15[14-l] + w7[6-l] (l <= 6): 15 multiply-adds instead of 22; then
// S = c3 + u and Sq = S + u (= S + c7 + c15). Window row j = x[t0 + r0 - 14 + j].
__device__ __forceinline__ void st_out(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_out(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <bool WQ, bool FULL, typename OT>
__device__ __forceinline__ void fwd_steps_merged(const float (&win)[WIN], const float (&b3)[3],
                                                 const float (&u)[15], OT* pS, OT* pQ,
                                                 int n, int D) {
#pragma unroll
  for (int i = 0; i < STEPS; ++i) {
    if (!FULL && i >= n) break;
    float s3 = 0.f, su = 0.f;
#pragma unroll
    for (int l = 2; l >= 0; --l) s3 += win[i + HALO - l] * b3[l];
#pragma unroll
    for (int l = 14; l >= 0; --l) su += win[i + HALO - l] * u[l];
    const float sum = s3 + su;
    st_out(pS, sum);
    pS += D;
    if (WQ) {
      st_out(pQ, sum + su);
      pQ += D;
    }
  }
}

// OT: output element type of S / Sq (float, or bf16 for the bf16 GEMM path,
// which needs no fp32 copy of S); c7 / c15 outputs exist for OT = float only.
template <bool WQ, bool WC, typename OT = float>
__global__ void __launch_bounds__(NW * 32, 3)
    conv_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w3,
                    const float* __restrict__ w7, const float* __restrict__ w15,
                    OT* __restrict__ S, OT* __restrict__ Sq, float* __restrict__ c7o,
                    float* __restrict__ c15o, int B, int T, int D, int nseg, int nparts) {
  rnet_dev::pdl_trigger();
  // persistent over tiles (b, segment) = p, p + nparts, ... of one channel
  // group, PIPE tiles in flight
  extern __shared__ __align__(16) float smem[];
  typedef float Tile[ROWS][CW];
  Tile* sx = reinterpret_cast<Tile*>(smem);  // [PIPE]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * CW;
  const int d = c0 + lane;
  const bool act = d < D;
  float a3[3], a7[7], a15[15];
#pragma unroll
  for (int k = 0; k < 3; ++k) a3[k] = act ? w3[k * D + d] : 0.f;
#pragma unroll
  for (int k = 0; k < 7; ++k) a7[k] = act ? w7[k * D + d] : 0.f;
#pragma unroll
  for (int k = 0; k < 15; ++k) a15[k] = act ? w15[k * D + d] : 0.f;
  float b3[3], u[15];  // per-lag taps of the merged path
#pragma unroll
  for (int l = 0; l < 3; ++l) b3[l] = a3[2 - l];
#pragma unroll
  for (int l = 0; l < 15; ++l) u[l] = a15[14 - l] + (l <= 6 ? a7[6 - l] : 0.f);
  const int r0 = warp * STEPS;  // window row j = x[t0 + r0 - HALO + j]
  const int items = B * nseg;
  auto stage_item = [&](int it, int buf) {
    if (it < items)
      stage(sx[buf], x, it / nseg, T, D, (it % nseg) * TS - HALO, c0);
    asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty
  };
#pragma unroll
  for (int q = 0; q < PIPE - 1; ++q) stage_item(blockIdx.y + q * nparts, q);
  int buf = 0;
  for (int it = blockIdx.y; it < items; it += nparts) {
    stage_item(it + (PIPE - 1) * nparts, (buf + PIPE - 1) % PIPE);
    asm volatile("cp.async.wait_group %0;" ::"n"(PIPE - 1) : "memory");
    __syncthreads();
    const int b = it / nseg;
    const int t0 = (it % nseg) * TS;
    if (act) {
      float win[WIN];
#pragma unroll
      for (int j = 0; j < WIN; ++j) win[j] = sx[buf][r0 + j][lane];
      const int tb = t0 + r0;
      const size_t o = ((size_t)b * T + tb) * D + d;
      const int n = T - tb < STEPS ? T - tb : STEPS;
      if constexpr (WC) {  // layer-op caches need c7 and c15 separately
        if (n == STEPS)
          fwd_steps<WQ, WC, true>(win, a3, a7, a15, S + o, Sq + o, c7o + o, c15o + o, STEPS, D);
        else if (n > 0)
          fwd_steps<WQ, WC, false>(win, a3, a7, a15, S + o, Sq + o, c7o + o, c15o + o, n, D);
      } else {
        if (n == STEPS)
          fwd_steps_merged<WQ, true, OT>(win, b3, u, S + o, Sq + o, STEPS, D);
        else if (n > 0)
          fwd_steps_merged<WQ, false, OT>(win, b3, u, S + o, Sq + o, n, D);
      }
    }
    __syncthreads();  // buffer `buf` is restaged PIPE - 1 iterations on
    buf = (buf + 1) % PIPE;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Data + weight gradient, merged by lag l = K-1-k (tap k of kernel K reads
// x[t - l]):
//   dx[t]   = sum_l E[l] dS[t + l],  E[l] = w15[14-l] + w7[6-l] + w3[2-l]
//             (terms present for l <= K-1): 15 multiply-adds per step, not 25;
//   C[l]   += x[t - l] dS[t], and dw_K[k] = sum C[K-1-k]: 15 lag correlations
//             per channel serve all 25 tap gradients.
// dx for one warp's steps from its dS window (gs[j] = dS[tb + j]); ACC: dx +=.
template <bool ACC, bool FULL>
__device__ __forceinline__ void dx_steps(const float (&gs)[WIN], const float (&E)[15], float* px,
                                         int n, int D) {
#pragma unroll
  for (int i = 0; i < STEPS; ++i) {
    if (!FULL && i >= n) break;
    float v = 0.f;
#pragma unroll
    for (int l = 14; l >= 0; --l) v += E[l] * gs[i + l];
    *px = ACC ? *px + v : v;
    px += D;
  }
}

// CTA (channel group, part p) loops over tiles (b, segment) = p, p + nparts,
// ...; dx rows of a tile need dS rows up to 14 steps AFTER it (anti-causal),
// the lag correlations x rows 14 steps before. Writes the CTA's 15 lag sums
// per channel to parts[p][15][D].
template <bool ACC>
__global__ void __launch_bounds__(NW * 32, 3)
    conv_bwd_kernel(const float* __restrict__ dS, const float* __restrict__ x,
                    const float* __restrict__ w3, const float* __restrict__ w7,
                    const float* __restrict__ w15, float* __restrict__ dx,
                    float* __restrict__ parts, int B, int T, int D, int nseg, int nparts) {
  rnet_dev::pdl_trigger();
  // PIPE_B buffers of {x tile, dS tile}: later tiles are staged while this one
  // is consumed
  extern __shared__ __align__(16) float smem[];
  typedef float Tile[ROWS][CW];
  Tile* sx = reinterpret_cast<Tile*>(smem);                     // [PIPE_B]
  Tile* sg = reinterpret_cast<Tile*>(smem + PIPE_B * ROWS * CW);  // [PIPE_B]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * CW;
  const int d = c0 + lane;
  const bool act = d < D;
  float E[15], C[15];
#pragma unroll
  for (int l = 0; l < 15; ++l) {
    float e = act ? w15[(14 - l) * D + d] : 0.f;
    if (l <= 6 && act) e += w7[(6 - l) * D + d];
    if (l <= 2 && act) e += w3[(2 - l) * D + d];
    E[l] = e;
    C[l] = 0.f;
  }
  const int r0 = warp * STEPS;
  const int items = B * nseg;
  auto stage_item = [&](int it, int buf) {
    if (it < items) {
      const int b = it / nseg;
      const int t0 = (it % nseg) * TS;
      stage(sx[buf], x, b, T, D, t0 - HALO, c0);  // row j = x[t0 - 14 + j]
      stage(sg[buf], dS, b, T, D, t0, c0);        // row j = dS[t0 + j]
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // possibly empty
  };
#pragma unroll
  for (int q = 0; q < PIPE_B - 1; ++q) stage_item(blockIdx.y + q * nparts, q);
  int buf = 0;
  for (int it = blockIdx.y; it < items; it += nparts) {
    stage_item(it + (PIPE_B - 1) * nparts, (buf + PIPE_B - 1) % PIPE_B);
    asm volatile("cp.async.wait_group %0;" ::"n"(PIPE_B - 1) : "memory");
    __syncthreads();
    const int b = it / nseg;
    const int t0 = (it % nseg) * TS;
    if (act) {
      float gs[WIN];  // dS[t0 + r0 + j]
#pragma unroll
      for (int j = 0; j < WIN; ++j) gs[j] = sg[buf][r0 + j][lane];
      const int tb = t0 + r0;
      const int n = T - tb < STEPS ? T - tb : STEPS;
      float* px = dx + ((size_t)b * T + tb) * D + d;
      if (n == STEPS)
        dx_steps<ACC, true>(gs, E, px, STEPS, D);
      else if (n > 0)
        dx_steps<ACC, false>(gs, E, px, n, D);
      // C[l] += x[t - l] dS[t] (dS zero past T). Window row j = x[t0 + r0 -
      // 14 + j] is read once and feeds every (l, i) with i + 14 - l = j; per
      // l the sum runs over i ascending.
#pragma unroll
      for (int j = 0; j < WIN; ++j) {
        const float xv = sx[buf][r0 + j][lane];
#pragma unroll
        for (int l = 0; l < 15; ++l) {
          const int i = j - 14 + l;
          if (i >= 0 && i < STEPS) C[l] += xv * gs[i];
        }
      }
    }
    __syncthreads();  // buffer `buf` is restaged PIPE_B - 1 iterations on
    buf = (buf + 1) % PIPE_B;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // CTA partial: sum the 8 warps' accumulators in warp order
  float(*red)[NW][CW] = reinterpret_cast<float(*)[NW][CW]>(smem);  // [15][8][32]
  static_assert(15 * NW * CW <= 2 * PIPE_B * ROWS * CW, "reduction scratch");
#pragma unroll
  for (int l = 0; l < 15; ++l) red[l][warp][lane] = C[l];
  __syncthreads();
  for (int l = warp; l < 15; l += NW) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) sum += red[l][w][lane];
    if (act) parts[((size_t)blockIdx.y * 15 + l) * D + d] = sum;
  }
}

// dw_K[k] += sum over parts of C[K-1-k] (parts in order; one lag sum serves
// the taps of every kernel size that reach it).
__global__ void conv_wgrad_reduce(const float* __restrict__ parts, int nparts, int D,
                                  float* __restrict__ dw3, float* __restrict__ dw7,
                                  float* __restrict__ dw15) {
  rnet_dev::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over 15*D
  if (i >= 15 * D) return;
  // loads in batches of 8 parts (independent), additions in part order
  float s = 0.f;
  for (int p0 = 0; p0 < nparts; p0 += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = p0 + j < nparts ? parts[(size_t)(p0 + j) * 15 * D + i] : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (p0 + j < nparts) s += v[j];
  }
  const int l = i / D, d = i % D;
  dw15[(14 - l) * D + d] += s;
  if (l <= 6) dw7[(6 - l) * D + d] += s;
  if (l <= 2) dw3[(2 - l) * D + d] += s;
}

// ---- TMA-pipelined backward (the model path) --------------------------------
// One persistent CTA per SM walks a contiguous range of the flattened tiles
// f = g * I + item (g = 64-channel group, item = (b, 128-step segment), I =
// items per group), so every SM gets the same number of tiles to within one.
// STAGES tiles are staged by TMA: the x tile (128 rows) and the dS tile (142
// rows: 14 steps past the tile, zero past T); lane 0 of warp 0 issues them,
// STAGES - 1 tiles ahead. A lane owns a channel pair (packed fp32 pairs).
// Warps 0-7 compute dx for 16 steps each; warps 8-15 the lag correlations of
// the same steps, taken forward in time,
//   C[l] = sum_t x[t] dS[t + l]  (= sum_t x[t - l] dS[t], dS zero past T),
// so x needs no halo. Splitting the two sums over separate warps halves each
// warp's dependent instruction stream and doubles the warps that hide its
// latency. When the range moves to the next channel group (and at the end)
// the correlation warps' C are summed in warp order into partial slot k + g
// (CTA k, group g: distinct for every intersecting pair), and
// conv_wgrad_reduce_slots sums each group's CTAs in CTA order.
namespace tb {
constexpr int CW = 64;                     // channels per tile (lane = pair)
constexpr int NW = 8;                      // warps per role (dx, correlations)
constexpr int THREADS = 2 * NW * 32;
constexpr int QS = 4;                      // dx steps per interleaved group
constexpr int RED_L = 3;                   // lags per reduction round
constexpr uint32_t RED_BYTES = RED_L * NW * CW * 4;
// STEPS steps per warp, STAGES tiles staged per CTA.
template <int STEPS_, int STAGES_>
struct Cfg {
  static constexpr int STEPS = STEPS_, STAGES = STAGES_;
  static constexpr int TS = NW * STEPS;            // steps per tile
  static constexpr int GROWS = TS + HALO;          // dS rows per tile
  static constexpr int WIN = STEPS + HALO;         // dS window per warp
  static constexpr uint32_t XBYTES = TS * CW * 4;
  static constexpr uint32_t GBYTES = GROWS * CW * 4;
  static constexpr uint32_t STAGE_BYTES = XBYTES + GBYTES;
  static constexpr size_t SMEM = 128 + STAGES * STAGE_BYTES + RED_BYTES + 64;
  static_assert(STAGE_BYTES % 128 == 0 && XBYTES % 128 == 0, "TMA destinations 128 B aligned");
  static_assert(STEPS % QS == 0, "step groups");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};
}  // namespace tb

// CTA holding flattened tile f when `total` tiles are split over P CTAs as
// [k * total / P, (k + 1) * total / P).
__host__ __device__ __forceinline__ int tile_owner(long long f, long long total, int P) {
  return (int)(((f + 1) * P + total - 1) / total) - 1;
}

// Barrier among the correlation warps only.
__device__ __forceinline__ void corr_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(tb::NW * 32) : "memory");
}

template <bool ACC, int STEPS_, int STAGES_>
__global__ void __launch_bounds__(tb::THREADS, 1)
    conv_bwd_tma_kernel(const __grid_constant__ CUtensorMap mX,
                        const __grid_constant__ CUtensorMap mG, const float* __restrict__ w3,
                        const float* __restrict__ w7, const float* __restrict__ w15,
                        float* __restrict__ dx, float* __restrict__ parts, int T, int D, int nseg,
                        int I, long long total, unsigned* err) {
  rnet_dev::pdl_trigger();
  using K = tb::Cfg<STEPS_, STAGES_>;
  constexpr int CW = tb::CW, NW = tb::NW, STEPS = K::STEPS, WIN = K::WIN, TS = K::TS;
  constexpr int STAGES = K::STAGES, RED_L = tb::RED_L, QS = tb::QS;
  constexpr uint32_t XBYTES = K::XBYTES, STAGE_BYTES = K::STAGE_BYTES, RED_BYTES = tb::RED_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  float* red = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);  // [RED_L][NW][CW]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + RED_BYTES);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool corr = warp >= NW;          // correlation warp (else dx warp)
  const int r0 = (warp % NW) * STEPS;
  const int P = gridDim.x, k = blockIdx.x;
  const long long f_lo = (long long)k * total / P, f_hi = (long long)(k + 1) * total / P;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2 * NW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const bool producer = threadIdx.x == 0;
  bool pok = true;  // producer still issuing
  // Stage tile number n of this CTA (after its stage's previous tile, n -
  // STAGES, has been released by every warp).
  auto issue = [&](int n) {
    const long long f = f_lo + n;
    if (!pok || f >= f_hi) return;
    const int s = n % STAGES;
    if (!mbar_wait(&empty[s], ((n / STAGES) & 1) ^ 1, err, abort_flag)) {
      pok = false;
      return;
    }
    const int g = (int)(f / I), it = (int)(f % I);
    uint8_t* st = smem + s * STAGE_BYTES;
    mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
    tma_load_3d(st, &mX, &full[s], g * CW, (it % nseg) * TS, it / nseg);
    tma_load_3d(st + XBYTES, &mG, &full[s], g * CW, (it % nseg) * TS, it / nseg);
  };
  if (producer) {
    tma_prefetch_desc(&mX);
    tma_prefetch_desc(&mG);
    for (int n = 0; n < STAGES - 1; ++n) issue(n);
  }

  uint64_t W[15];  // dx warps: merged taps E[l]; correlation warps: C[l]
  int cur_g = -1;
  bool ok = true;
  // Correlation warps: sum their C in warp order into slot k + g (each runs
  // the same sequence of flushes, also after a failed wait).
  auto flush = [&](int g) {
    const int ct = threadIdx.x - NW * 32;  // thread index among correlation warps
#pragma unroll
    for (int l0 = 0; l0 < 15; l0 += RED_L) {
      corr_sync();  // the previous round's readers are done
#pragma unroll
      for (int q = 0; q < RED_L; ++q)
        reinterpret_cast<uint64_t*>(red)[(q * NW + warp - NW) * (CW / 2) + lane] = W[l0 + q];
      corr_sync();
      if (ct < RED_L * CW) {
        const int q = ct / CW, cc = ct % CW;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += red[(q * NW + w) * CW + cc];
        if (g * CW + cc < D) parts[((size_t)(k + g) * 15 + l0 + q) * CW + cc] = sum;
      }
    }
  };
  int n = 0;
  for (long long f = f_lo; f < f_hi; ++f, ++n) {
    if (producer) issue(n + STAGES - 1);
    __syncwarp();
    const int g = (int)(f / I), it = (int)(f % I);
    const int d = g * CW + 2 * lane;  // channels d, d + 1 (D % 4 == 0: both or neither)
    const bool act = d < D;
    if (g != cur_g) {
      if (corr) {
        if (cur_g >= 0) flush(cur_g);
#pragma unroll
        for (int l = 0; l < 15; ++l) W[l] = 0;
      } else {
#pragma unroll
        for (int l = 0; l < 15; ++l) {
          float e0 = 0.f, e1 = 0.f;
          if (act) {
            e0 = w15[(14 - l) * D + d];
            e1 = w15[(14 - l) * D + d + 1];
            if (l <= 6) {
              e0 += w7[(6 - l) * D + d];
              e1 += w7[(6 - l) * D + d + 1];
            }
            if (l <= 2) {
              e0 += w3[(2 - l) * D + d];
              e1 += w3[(2 - l) * D + d + 1];
            }
          }
          W[l] = pk_make(e0, e1);
        }
      }
      cur_g = g;
    }
    const int s = n % STAGES;
    ok = ok && mbar_wait(&full[s], (n / STAGES) & 1, err, abort_flag);
    if (ok) {
      const uint64_t* sx = reinterpret_cast<const uint64_t*>(smem + s * STAGE_BYTES);
      const uint64_t* sg = reinterpret_cast<const uint64_t*>(smem + s * STAGE_BYTES + XBYTES);
      uint64_t gs[WIN];  // dS[tb + j], channel pair of this lane
#pragma unroll
      for (int j = 0; j < WIN; ++j) gs[j] = sg[(r0 + j) * (CW / 2) + lane];
      if (corr) {
#pragma unroll
        for (int i = 0; i < STEPS; ++i) {
          const uint64_t xv = sx[(r0 + i) * (CW / 2) + lane];  // zero past T
#pragma unroll
          for (int l = 0; l < 15; ++l) W[l] = pk_fma(xv, gs[i + l], W[l]);
        }
      } else {
        const int b = it / nseg, tb = (it % nseg) * TS + r0;
        const int nv = T - tb;  // valid steps of this warp (may be <= 0)
        uint64_t* px = reinterpret_cast<uint64_t*>(dx + ((size_t)b * T + tb) * D + d);
        // QS independent dx chains at a time
#pragma unroll
        for (int i0 = 0; i0 < STEPS; i0 += QS) {
          uint64_t v[QS], prev[ACC ? QS : 1];  // ACC: the group's dx rows, loaded first
          if (ACC) {
#pragma unroll
            for (int q = 0; q < QS; ++q)
              prev[ACC ? q : 0] = act && i0 + q < nv ? px[(size_t)(i0 + q) * (D / 2)] : 0;
          }
#pragma unroll
          for (int q = 0; q < QS; ++q) v[q] = 0;
#pragma unroll
          for (int l = 14; l >= 0; --l) {
#pragma unroll
            for (int q = 0; q < QS; ++q) v[q] = pk_fma(W[l], gs[i0 + q + l], v[q]);
          }
#pragma unroll
          for (int q = 0; q < QS; ++q) {
            const int i = i0 + q;
            if (act && i < nv) {
              uint64_t* p = px + (size_t)i * (D / 2);
              *p = ACC ? pk_add(prev[ACC ? q : 0], v[q]) : v[q];
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (corr && cur_g >= 0) flush(cur_g);
}

// dw_K[k] += sum over the CTAs that worked on channel group g of their lag
// sums (slot k + g, CTAs in order).
__global__ void conv_wgrad_reduce_slots(const float* __restrict__ parts, int D, int I,
                                        long long total, int P, float* __restrict__ dw3,
                                        float* __restrict__ dw7, float* __restrict__ dw15) {
  rnet_dev::pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // over 15*D
  if (i >= 15 * D) return;
  const int l = i / D, d = i % D, g = d / tb::CW, cc = d % tb::CW;
  const int k0 = tile_owner((long long)g * I, total, P);
  const int k1 = tile_owner((long long)g * I + I - 1, total, P);
  float s = 0.f;
  for (int kk = k0; kk <= k1; kk += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = kk + j <= k1 ? parts[((size_t)(kk + j + g) * 15 + l) * tb::CW + cc] : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (kk + j <= k1) s += v[j];
  }
  dw15[(14 - l) * D + d] += s;
  if (l <= 6) dw7[(6 - l) * D + d] += s;
  if (l <= 2) dw3[(2 - l) * D + d] += s;
}

int nparts_for(int B, int T, int D) {
  const int nseg = (T + TS - 1) / TS;
  const int groups = (D + CW - 1) / CW;
  int p = (148 * 3) / groups;  // every CTA resident (three per SM)
  if (p > MAX_PARTS) p = MAX_PARTS;
  if (p > B * nseg) p = B * nseg;
  return p < 1 ? 1 : p;
}

}  // namespace

cudaError_t conv_fwd(const float* x, const float* w3, const float* w7, const float* w15, float* S,
                     float* Sq, float* c7, float* c15, int B, int T, int D, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 4) return cudaErrorInvalidValue;
  const int nseg = (T + TS - 1) / TS;
  const int groups = (D + CW - 1) / CW;
  // persistent: three CTAs per SM (<= 85 registers x 256 threads, 55 KB each)
  int np = (148 * 3) / groups;
  if (np > B * nseg) np = B * nseg;
  if (np < 1) np = 1;
  // Sq (model path) and c7/c15 (layer-op caches) are never asked for together
  if ((c7 == nullptr) != (c15 == nullptr) || (Sq && c7)) return cudaErrorInvalidValue;
  constexpr size_t smem = PIPE * ROWS * CW * sizeof(float);
  auto kern = Sq ? conv_fwd_kernel<true, false>
                 : (c7 ? conv_fwd_kernel<false, true> : conv_fwd_kernel<false, false>);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(groups, np);
  kern<<<grid, NW * 32, smem, s>>>(x, w3, w7, w15, S, Sq, c7, c15, B, T, D, nseg, np);
  return launched();
}

cudaError_t conv_fwd_bf16(const float* x, const float* w3, const float* w7, const float* w15,
                          __nv_bfloat16* S16, __nv_bfloat16* Sq16, int B, int T, int D,
                          cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 4 || !S16) return cudaErrorInvalidValue;
  const int nseg = (T + TS - 1) / TS;
  const int groups = (D + CW - 1) / CW;
  int np = (148 * 3) / groups;
  if (np > B * nseg) np = B * nseg;
  if (np < 1) np = 1;
  constexpr size_t smem = PIPE * ROWS * CW * sizeof(float);
  auto kern = Sq16 ? conv_fwd_kernel<true, false, __nv_bfloat16>
                   : conv_fwd_kernel<false, false, __nv_bfloat16>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(groups, np);
  kern<<<grid, NW * 32, smem, s>>>(x, w3, w7, w15, S16, Sq16, nullptr, nullptr, B, T, D, nseg,
                                   np);
  return launched();
}

size_t conv_bwd_partials_floats(int B, int T, int D) {
  const size_t v1 = (size_t)nparts_for(B, T, D) * 15 * D;
  // TMA path: slots k + g, k < SMs, g < channel groups
  const size_t v2 = (size_t)(rnet_gemm::num_sms() + (D + tb::CW - 1) / tb::CW) * 15 * tb::CW;
  return v1 > v2 ? v1 : v2;
}

namespace {

// The TMA path needs 16-byte aligned dS, x and dx (tensor-map bases, packed
// stores); RNET_CONV_BWD_TILED=1 forces the cp.async path (A/B timing).
bool tma_path_enabled() {
  static const bool on = [] {
    const char* e = getenv("RNET_CONV_BWD_TILED");
    return !(e && e[0] == '1');
  }();
  return on;
}

template <bool ACC, int STEPS, int STAGES>
cudaError_t launch_bwd_tma(const float* dS, const float* x, const float* w3, const float* w7,
                           const float* w15, float* dx, float* dw3, float* dw7, float* dw15,
                           float* parts, int B, int T, int D, cudaStream_t s, bool* done) {
  using K = tb::Cfg<STEPS, STAGES>;
  *done = false;
  const int nseg = (T + K::TS - 1) / K::TS;
  const int G = (D + tb::CW - 1) / tb::CW;
  const int I = B * nseg;
  const long long total = (long long)G * I;
  const int P = (int)(total < rnet_gemm::num_sms() ? total : rnet_gemm::num_sms());
  const uint64_t dims[3] = {(uint64_t)D, (uint64_t)T, (uint64_t)B};
  const uint64_t strides[2] = {(uint64_t)D * 4, (uint64_t)T * D * 4};
  const uint32_t box_x[3] = {tb::CW, (uint32_t)K::TS, 1};
  const uint32_t box_g[3] = {tb::CW, (uint32_t)K::GROWS, 1};
  CUtensorMap mX, mG;
  if (!rnet_gemm::encode_map_f32(&mX, x, 3, dims, strides, box_x) ||
      !rnet_gemm::encode_map_f32(&mG, dS, 3, dims, strides, box_g))
    return cudaSuccess;  // not encodable: the caller takes the cp.async path
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(conv_bwd_tma_kernel<ACC, STEPS, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)K::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  conv_bwd_tma_kernel<ACC, STEPS, STAGES><<<P, tb::THREADS, K::SMEM, s>>>(
      mX, mG, w3, w7, w15, dx, parts, T, D, nseg, I, total, rnet_status::device_error_word());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  conv_wgrad_reduce_slots<<<(15 * D + 255) / 256, 256, 0, s>>>(parts, D, I, total, P, dw3, dw7,
                                                               dw15);
  *done = true;
  return launched(2);
}

}  // namespace

cudaError_t conv_bwd(const float* dS, const float* x, const float* w3, const float* w7,
                     const float* w15, float* dx, float* dw3, float* dw7, float* dw15,
                     float* partials, int B, int T, int D, int accumulate, cudaStream_t s) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  if (D % 4) return cudaErrorInvalidValue;
  const bool aligned = ((reinterpret_cast<uintptr_t>(dS) | reinterpret_cast<uintptr_t>(x) |
                         reinterpret_cast<uintptr_t>(dx)) & 15) == 0;
  if (aligned && tma_path_enabled()) {
    bool done = false;
    cudaError_t e;
    // 128-step tiles, 3 stages (64-step tiles with 5 stages measured slower)
    e = accumulate ? launch_bwd_tma<true, 16, 3>(dS, x, w3, w7, w15, dx, dw3, dw7, dw15, partials,
                                                 B, T, D, s, &done)
                   : launch_bwd_tma<false, 16, 3>(dS, x, w3, w7, w15, dx, dw3, dw7, dw15, partials,
                                                  B, T, D, s, &done);
    if (e != cudaSuccess || done) return e;
  }
  const int nseg = (T + TS - 1) / TS;
  const int np = nparts_for(B, T, D);
  dim3 grid((D + CW - 1) / CW, np);
  constexpr size_t smem = 2 * PIPE_B * ROWS * CW * sizeof(float);
  auto kern = accumulate ? conv_bwd_kernel<true> : conv_bwd_kernel<false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, NW * 32, smem, s>>>(dS, x, w3, w7, w15, dx, partials, B, T, D, nseg, np);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  conv_wgrad_reduce<<<(15 * D + 255) / 256, 256, 0, s>>>(partials, np, D, dw3, dw7, dw15);
  return launched(2);
}

}  // namespace rnet_k
