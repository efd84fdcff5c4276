// Persistent warp-specialised tcgen05 GEMM for sm_100a with 3xTF32 error
// compensation, so fp32 operands give fp32-class results on the tensor cores.
//
// A tf32 operand read keeps the top 19 bits of an fp32 word (the low 13
// mantissa bits are ignored), so the raw fp32 tile already IS the "hi" part.
// Split warps only compute lo = x - (x with the low 13 bits cleared) into a
// twin buffer; each 8-deep K slice then issues three kind::tf32 UMMAs
// (hi*lo, lo*hi, hi*hi) into one fp32 TMEM accumulator. The dropped lo*lo
// term is ~2^-22 relative.
//
// Roles (448 threads = 14 warps):
//   warps 0-3  epilogue (warp w owns TMEM lanes 32w..32w+31 = tile rows)
//   warp  4    TMA producer (raw fp32 tiles)
//   warp  5    TMEM allocator + single-thread UMMA issuer
//   warps 6-13 split warps (lo = x - trunc_tf32(x) into the twin buffer)
// Pipelines: full[s] (TMA tx) -> split[s] (8 warp arrivals) -> empty[s]
// (tcgen05.commit); accumulators double-buffered in TMEM with accf/acce.
//
// K-blocks are 16 fp32 deep (64-byte rows, SWIZZLE_64B for K-major operands,
// SWIZZLE_128B_ATOM_32B boxes of 32 x 16 for MN-major ones), which fits 4
// pipeline stages at BN = 256 (6 at BN = 128): the pipeline is latency-bound
// with fewer stages.
//
// Reference parity: replaces every cublasSgemm call of the reference
// (src/min_gru.cu:64-178, src/causal_conv.cu:76-165, src/slot_memory.cu:91-235,
// src/swiglu_ffn.cu:32-143, src/embedding.cu:61, src/resonance_net.cpp:428-437).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include <cuda_bf16.h>

#include "common.cuh"
#include "conv_step.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

namespace rnet_gemm {
using namespace rnet_dev;

constexpr int BM = 128;
constexpr int NUM_EPI_WARPS = 4;
constexpr int PRODUCER_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr int FIRST_SPLIT_WARP = 6;
constexpr int NUM_SPLIT_WARPS = 8;
constexpr int NUM_THREADS = 32 * (FIRST_SPLIT_WARP + NUM_SPLIT_WARPS);
constexpr int SMEM_BUDGET = 200 * 1024;  // pipeline stages (barriers etc. extra)
constexpr int TILE_LD = 33;              // epilogue transpose tile: 32 x 33 floats per warp
// per-warp epilogue slot: a 32 x 33 transpose tile, or two 32 x 32 fp32 tiles
// in the SWIZZLE_128B layout a TMA store reads (slots 1024-byte aligned), used
// alternately so one tile's copy overlaps the next tile's TMEM load and
// shared-memory writes (one buffer: the copies ran back to back, 3.3 of a
// short-K decode GEMM's 8.5 us)
constexpr int EPI_TILE_FLOATS = 2048;
static_assert(EPI_TILE_FLOATS >= 32 * TILE_LD && (EPI_TILE_FLOATS * 4) % 1024 == 0, "epi slot");

struct KParams {
  int M, N, K;
  int m_tiles, n_tiles, k_splits, kb_total, kb_per_split;
  int num_units;
  int row_owner;   // 1: a unit is one m-tile swept over all n-tiles
  int b_pair_off;  // rows
  int a_mn, b_mn;
  // split-K into a workspace: split ks stores its partial at epi.C + ks *
  // split_stride (0: no workspace split)
  long long split_stride;
  // 1: store / accumulate / residual tiles go through the warp's shared-memory
  // tile (TMA bulk store / reduce-add, or coalesced 128-byte rows) instead of
  // thread-per-row stores (32 lines per instruction): always with bf16 tiles,
  // with fp32 tiles when TMA stores them. Measured: config-2 fp32 step
  // 15.47 -> 14.62 ms, bf16 GEMM M16384 N2048 K512 77.5 -> 42.8 us.
  int stage_epi;
  // 1: store / accumulate tiles leave through TMA (bulk tensor store or
  // reduce-add of each warp's 32 x 32 tile from shared memory), the store
  // map being the kernel's tmC
  int tma_out;
  // SwiGLU forward: 2 or 3 when G, U (and H) are planes of one 3-D tensor
  // map (tmC: [planes][M][ldf]) that TMA stores; 0 = warp stores
  int swiglu_planes;
  // 1 when the bf16 copy (SwiGLU forward's H16, a store's C16) leaves through
  // TMA (tmD: bf16 rows, 32 x 32 boxes) instead of the warp's transpose tile
  int copy16_tma;
  Epilogue epi;
  unsigned* err;
};

// BN = MMA N (accumulator columns per tile). CG = 2: one MMA covers the
// 2*BM rows of a CTA pair; each CTA stages its BM rows of A and BN/2 rows of B.
// ELEM = bytes per staged element (4: fp32 tiles; 2: bf16 tiles read straight
// from bf16 operands), LO = a twin buffer per stage (the split warps' lo or
// bf16 tiles).
template <int BN, int BK, int CG, int ELEM = 4, bool LO = true, int NEPI = NUM_EPI_WARPS>
struct Cfg {
  static constexpr int ROW_BYTES = BK * ELEM;         // K-major row (64 or 128 B)
  static constexpr int MN_ELEMS = 128 / ELEM;         // MN-major box width (one 128 B row)
  static constexpr int MN_CHUNK = 128 * BK;           // MN-major box: MN_ELEMS x BK rows
  static constexpr int B_ROWS = BN / CG;              // B rows staged by this CTA
  static constexpr int A_BYTES = BM * BK * ELEM;
  static constexpr int B_BYTES = B_ROWS * BK * ELEM;
  static constexpr int RAW_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = LO ? 2 * RAW_BYTES : RAW_BYTES;  // raw (= hi) + lo
  static constexpr int EPI_BYTES = NEPI * EPI_TILE_FLOATS * 4;
  // more epilogue warps take their tiles out of the stage budget
  static constexpr int STAGES_BUDGET =
      (SMEM_BUDGET - (NEPI - NUM_EPI_WARPS) * EPI_TILE_FLOATS * 4) / STAGE_BYTES;
  static constexpr int STAGES_LIMIT = (227 * 1024 - EPI_BYTES - 1024 - 256) / STAGE_BYTES;
  static constexpr int STAGES_FIT = STAGES_BUDGET < STAGES_LIMIT ? STAGES_BUDGET : STAGES_LIMIT;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
  // UMMA smem-descriptor parameters
  static constexpr uint32_t K_LAYOUT = ROW_BYTES == 128 ? 2u : 4u;  // SWIZZLE_128B / _64B
  static constexpr uint32_t K_SBO = 8 * ROW_BYTES;          // 8-row core-matrix group
  static_assert((ELEM == 4 && (BK == 16 || BK == 32)) || (ELEM == 2 && BK == 64), "BK");
  static_assert(CG == 1 || CG == 2, "CG");
  static_assert(STAGES >= 2, "stages");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory above the per-CTA opt-in limit");
  static_assert(B_ROWS % MN_ELEMS == 0, "B rows");
};

__device__ __forceinline__ void unit_range(const KParams& p, int unit, int& mt, int& nt0,
                                           int& nt1, int& kb0, int& kb1) {
  if (p.row_owner) {
    mt = unit;
    nt0 = 0;
    nt1 = p.n_tiles;
    kb0 = 0;
    kb1 = p.kb_total;
  } else {
    const int nt = unit % p.n_tiles;
    const int rest = unit / p.n_tiles;
    const int ks = rest % p.k_splits;
    mt = rest / p.k_splits;
    nt0 = nt;
    nt1 = nt + 1;
    kb0 = ks * p.kb_per_split;
    kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  }
}


// ------------------------------------------------------------------ epilogue
// The accumulator arrives thread-per-row (TMEM lane = tile row, 32 columns
// per tcgen05.ld). The SwiGLU forward epilogue, which writes three [N, F]
// planes per tile, goes through a per-warp 32x33 shared-memory tile so that a warp
// instruction touches four full 128-byte row segments (coalesced float4)
// instead of 32 rows; the other kinds store thread-per-row directly.
// Thread `lane` holds row (row0 + lane) x columns [col0, col0 + 32) in v.
// Writes the 32x32 block to dst (row stride ld) with coalesced float4 stores:
// op 0 = store, 1 = red.add, 2 = store R + v (R row stride ldr).
__device__ __forceinline__ void tile_out(float* st, const float (&v)[32], float* dst, int ld,
                                         const float* R, int ldr, int row0, int col0, int M,
                                         int N, int op, __nv_bfloat16* dst16 = nullptr) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 32; ++i) st[lane * TILE_LD + i] = v[i];
  __syncwarp();
  const int cc = (lane & 7) * 4;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int rr = j * 4 + (lane >> 3);
    const int row = row0 + rr, col = col0 + cc;
    if (row < M) {
      const float* s = st + rr * TILE_LD + cc;
      float4 x = make_float4(s[0], s[1], s[2], s[3]);
      float* g = dst + (size_t)row * ld + col;
      if (col + 4 <= N) {
        if (op == 1) {
          red_add_v4(g, x.x, x.y, x.z, x.w);
        } else {
          if (op == 2) {
            const float4 r = *reinterpret_cast<const float4*>(R + (size_t)row * ldr + col);
            x.x += r.x; x.y += r.y; x.z += r.z; x.w += r.w;
          }
          if (dst) *reinterpret_cast<float4*>(g) = x;
          if (dst16) {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(x.x, x.y);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(x.z, x.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&lo);
            u.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(dst16 + (size_t)row * ld + col) = u;
          }
        }
      } else {
        const float xs[4] = {x.x, x.y, x.z, x.w};
        for (int q = 0; q < 4 && col + q < N; ++q) {
          if (op == 1) {
            atomicAdd(g + q, xs[q]);
          } else {
            const float o = xs[q] + (op == 2 ? R[(size_t)row * ldr + col + q] : 0.f);
            if (dst) g[q] = o;
            if (dst16) dst16[(size_t)row * ld + col + q] = __float2bfloat16_rn(o);
          }
        }
      }
    }
  }
  __syncwarp();
}

// 32 consecutive values a * v[i] as bf16 (four 16-byte stores).
__device__ __forceinline__ void store_bf16_row32(__nv_bfloat16* dst, const float (&v)[32], float a,
                                                 const void*) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(a * v[8 * j + 2 * i], a * v[8 * j + 2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    u.x = w[0]; u.y = w[1]; u.z = w[2]; u.w = w[3];
    reinterpret_cast<uint4*>(dst)[j] = u;
  }
}

// Direct thread-per-row store of one 32-column chunk (row stride ld): eight
// float4 per thread. For plain stores / split-K reductions / residual adds
// this beats staging through shared memory, which competes with the
// operand pipeline for shared-memory bandwidth.
__device__ __forceinline__ void store_row_chunk(const KParams& p, int kind, int row, int col0,
                                                const float (&v)[32], size_t c_off = 0) {
  Epilogue e = p.epi;
  e.C += c_off;
  if (row >= p.M) return;
  const float a = e.alpha;
  if (col0 + 32 <= p.N) {
    if (kind == EPI_STORE) {
      float4* dst = reinterpret_cast<float4*>(e.C + (size_t)row * e.ldc + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dst[j] = make_float4(a * v[4 * j], a * v[4 * j + 1], a * v[4 * j + 2], a * v[4 * j + 3]);
      if (e.C16) store_bf16_row32(e.C16 + (size_t)row * e.ldc + col0, v, a, nullptr);
    } else if (kind == EPI_ACCUM) {
      float* dst = e.C + (size_t)row * e.ldc + col0;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        red_add_v4(dst + 4 * j, a * v[4 * j], a * v[4 * j + 1], a * v[4 * j + 2],
                   a * v[4 * j + 3]);
    } else {  // EPI_RESID
      const float4* r = reinterpret_cast<const float4*>(e.R + (size_t)row * e.ldr + col0);
      float4* dst = reinterpret_cast<float4*>(e.C + (size_t)row * e.ldc + col0);
      float o[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 q = r[j];
        o[4 * j] = q.x + a * v[4 * j];
        o[4 * j + 1] = q.y + a * v[4 * j + 1];
        o[4 * j + 2] = q.z + a * v[4 * j + 2];
        o[4 * j + 3] = q.w + a * v[4 * j + 3];
        dst[j] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      }
      if (e.C16) store_bf16_row32(e.C16 + (size_t)row * e.ldc + col0, o, 1.0f, nullptr);
    }
  } else {
    for (int i = 0; i < 32; ++i) {
      const int col = col0 + i;
      if (col < p.N) {
        float* dst = e.C + (size_t)row * e.ldc + col;
        if (kind == EPI_STORE) *dst = a * v[i];
        else if (kind == EPI_ACCUM) atomicAdd(dst, a * v[i]);
        else *dst = e.R[(size_t)row * e.ldr + col] + a * v[i];
        if (e.C16 && kind != EPI_ACCUM)
          e.C16[(size_t)row * e.ldc + col] = __float2bfloat16_rn(*dst);
      }
    }
  }
}

// The residual rows the epilogue reads for the warp's 32 rows x BN columns of
// tile nt, prefetched into L2 while the tile's MMAs still run, so the
// epilogue's loads hit L2 instead of DRAM.
template <int BN>
__device__ __forceinline__ void prefetch_epilogue_inputs(const KParams& p, int row, int nt) {
  const Epilogue& e = p.epi;
  if (row >= p.M) return;
  if (e.kind == EPI_RESID) {
    const int c0 = nt * BN;
#pragma unroll
    for (int c = 0; c < BN; c += 32)
      if (c0 + c < p.N) prefetch_l2(e.R + (size_t)row * e.ldr + c0 + c);
  }
}

// Bulk tensor store / reduce-add of one 32 x 32 fp32 tile (SWIZZLE_128B in
// shared memory) to (x = col, y = row) of the map; bulk-group completion.
__device__ __forceinline__ void tma_store_tile(const void* map, const void* smem, int x, int y,
                                               bool reduce_add) {
  if (reduce_add)
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], "
        "[%3];" ::"l"(map), "r"(x), "r"(y), "r"(smem_u32(smem))
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
        "r"(x), "r"(y), "r"(smem_u32(smem))
        : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// 3-D form (z = plane) for the SwiGLU outputs.
__device__ __forceinline__ void tma_store_tile3(const void* map, const void* smem, int x, int y,
                                                int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          map),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem))
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// The warp's next 32 x 32 TMA staging buffer (alternating halves of its
// slot): free once at most one bulk group, the other half's, is still
// reading. The caller's sub-tile ends with bulk_wait_read_all().
__device__ __forceinline__ float* tma_stage_next(float* slot, int& n, int lane) {
  float* b = slot + (n & 1) * 1024;
  ++n;
  if (lane == 0) bulk_wait_read_1();
  __syncwarp();
  return b;
}

// A 32 x 32 bf16 tile (lane = row, 64 B per row, no swizzle) from fp32
// values, rounded to nearest even, ready for a TMA store through tmD.
__device__ __forceinline__ void stage_bf16_tile(float* buf, const float (&v)[32], int lane) {
  uint4* t = reinterpret_cast<uint4*>(buf);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * j + 2 * i], v[8 * j + 2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    t[lane * 4 + j] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
}

struct Top2State {
  float h0, h1;
  int i0, i1;
};

// One accumulator sub-tile (128 rows x BN columns); warp q handles rows
// row0 = m0 + 32q .. +31, `st` is the warp's smem tile.
// cfirst / cstep: this warp's share of the 32-column chunks when several
// warps serve one TMEM lane quadrant (store / accumulate / residual kinds
// only; the SwiGLU and top-2 kinds run on the cfirst == 0 warp).
template <int BN, bool PIPE_LD>
__device__ __forceinline__ void epilogue_subtile(const KParams& p, uint32_t tacc, int row0,
                                                 int nt, bool last_sub, Top2State& st,
                                                 float* tile, size_t c_off, int cfirst = 0,
                                                 int cstep = 1, const void* tmC = nullptr,
                                                 const void* tmD = nullptr) {
  const Epilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  const int row = row0 + lane;
  float v[32];
  if (e.kind == EPI_TOP2 && cfirst != 0) return;
  if (e.kind == EPI_SWIGLU_FWD) {
    constexpr int HALF_CHUNKS = BN / 64;
    // one 32 x 32 tile through TMA: swizzled into the warp's slot, stored
    // as plane z (the slot is free again once the copy has read it)
    int nbuf = 0;
    auto tma_plane = [&](const float (&x)[32], int f0, int z) {
      float* buf = tma_stage_next(tile, nbuf, lane);
      float4* t4 = reinterpret_cast<float4*>(buf);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        t4[lane * 8 + (j ^ (lane & 7))] =
            make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tma_store_tile3(tmC, buf, f0, row0, z);
    };
#pragma unroll 1
    for (int c = cfirst; c < HALF_CHUNKS; c += cstep) {
      float g[32];
      tmem_ld_32cols(tacc + c * 32, g);
      tmem_ld_32cols(tacc + (c + HALF_CHUNKS) * 32, v);
      const int f0 = nt * (BN / 2) + c * 32;
      if (p.swiglu_planes) {
        tma_plane(g, f0, 0);
        tma_plane(v, f0, 1);
      } else {
        tile_out(tile, g, e.G, e.ldf, nullptr, 0, row0, f0, p.M, p.N, 0);
        tile_out(tile, v, e.U, e.ldf, nullptr, 0, row0, f0, p.M, p.N, 0);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = silu_fast(g[i]) * v[i];
      if (p.swiglu_planes == 3) {
        tma_plane(v, f0, 2);
      } else if (p.copy16_tma) {
        // bf16 H in the next staging buffer
        float* buf = tma_stage_next(tile, nbuf, lane);
        stage_bf16_tile(buf, v, lane);
        if (lane == 0) tma_store_tile(tmD, buf, f0, row0, false);
      } else {
        if (p.swiglu_planes) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
        tile_out(tile, v, e.H, e.ldf, nullptr, 0, row0, f0, p.M, p.N, 0, e.H16);
      }
    }
    if (p.swiglu_planes) {
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
    }
    return;
  }
  if (e.kind == EPI_TOP2) {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      tmem_ld_32cols(tacc + c * 32, v);
      const int s0 = nt * BN + c * 32;
      if (e.C != nullptr) store_row_chunk(p, EPI_STORE, row, s0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s = s0 + i;
        const float x = v[i] * e.alpha;
        // Reference order (src/slot_memory.cu:40-51): replace the first
        // minimum of the held pair when strictly greater.
        const bool m1 = st.h1 < st.h0;
        const float hm = m1 ? st.h1 : st.h0;
        if (s < p.N && x > hm) {
          if (m1) { st.h1 = x; st.i1 = s; } else { st.h0 = x; st.i0 = s; }
        }
      }
    }
    if (last_sub && row < p.M) {
      const float mx = fmaxf(st.h0, st.h1);
      const float e0 = __expf(st.h0 - mx), e1 = __expf(st.h1 - mx);
      const float sum = e0 + e1;
      e.topk_idx[2 * (size_t)row] = st.i0;
      e.topk_idx[2 * (size_t)row + 1] = st.i1;
      e.topk_w[2 * (size_t)row] = e0 / sum;
      e.topk_w[2 * (size_t)row + 1] = e1 / sum;
    }
    return;
  }
  if (p.stage_epi) {
    const int op = e.kind == EPI_STORE ? 0 : (e.kind == EPI_ACCUM ? 1 : 2);
    const bool tma = p.tma_out && ((op == 0 && (e.C16 == nullptr || p.copy16_tma)) || op == 1);
    if (PIPE_LD && tma && e.C16 == nullptr) {
      // the next chunk's TMEM load is in flight while this chunk is staged
      // and its bulk copy issued (fp32 tiles: decode step 0.531 -> 0.520 ms;
      // bf16 storage keeps the plain loop, which spills less: 7.39 -> 7.23 ms)
      const int plane = p.tma_out == 2 ? (int)(c_off / p.split_stride) : 0;
      int nbuf = 0;
      uint32_t cur[32], nxt[32];
      if (cfirst < BN / 32) {
        tmem_ld_32cols_issue(tacc + cfirst * 32, cur);
        tmem_ld_wait(cur);
      }
#pragma unroll 1
      for (int c = cfirst; c < BN / 32; c += cstep) {
        const bool more = c + cstep < BN / 32;
        if (more) tmem_ld_32cols_issue(tacc + (c + cstep) * 32, nxt);
        float* buf = tma_stage_next(tile, nbuf, lane);
        float4* t4 = reinterpret_cast<float4*>(buf);
        const float al = e.alpha;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          t4[lane * 8 + (j ^ (lane & 7))] =
              make_float4(al * __uint_as_float(cur[4 * j]), al * __uint_as_float(cur[4 * j + 1]),
                          al * __uint_as_float(cur[4 * j + 2]),
                          al * __uint_as_float(cur[4 * j + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (p.tma_out == 2)  // split-K partial: plane = split index
            tma_store_tile3(tmC, buf, nt * BN + c * 32, row0, plane);
          else
            tma_store_tile(tmC, buf, nt * BN + c * 32, row0, op == 1);
        }
        if (more) {
          tmem_ld_wait(nxt);
#pragma unroll
          for (int i = 0; i < 32; ++i) cur[i] = nxt[i];
        }
      }
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
      return;
    }
    int nbuf = 0;
#pragma unroll 1
    for (int c = cfirst; c < BN / 32; c += cstep) {
      tmem_ld_32cols(tacc + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= e.alpha;
      if (tma) {
        float* buf = tma_stage_next(tile, nbuf, lane);
        float4* t4 = reinterpret_cast<float4*>(buf);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          t4[lane * 8 + (j ^ (lane & 7))] =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (p.tma_out == 2)  // split-K partial: plane = split index
            tma_store_tile3(tmC, buf, nt * BN + c * 32, row0, (int)(c_off / p.split_stride));
          else
            tma_store_tile(tmC, buf, nt * BN + c * 32, row0, op == 1);
        }
        if (e.C16 != nullptr && op == 0) {  // the bf16 copy through tmD
          float* b16 = tma_stage_next(tile, nbuf, lane);
          stage_bf16_tile(b16, v, lane);
          if (lane == 0) tma_store_tile(tmD, b16, nt * BN + c * 32, row0, false);
        }
      } else {
        tile_out(tile, v, e.C + c_off, e.ldc, e.R, e.ldr, row0, nt * BN + c * 32, p.M, p.N, op,
                 op == 1 ? nullptr : e.C16);
      }
    }
    if (tma) {
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
    }
    return;
  }
  // residual: this thread's 32-column slice of row `row` is one 128-byte
  // line; the next chunk's line is pulled into L1 while this one is stored
  const bool resid = e.kind == EPI_RESID && row < p.M;
  const float* rrow = e.R + (size_t)row * e.ldr + nt * BN;
  if (resid && nt * BN + cfirst * 32 < p.N) prefetch_l1(rrow + cfirst * 32);
#pragma unroll 1
  for (int c = cfirst; c < BN / 32; c += cstep) {
    if (resid && c + cstep < BN / 32 && nt * BN + (c + cstep) * 32 < p.N)
      prefetch_l1(rrow + (c + cstep) * 32);
    tmem_ld_32cols(tacc + c * 32, v);
    store_row_chunk(p, e.kind, row, nt * BN + c * 32, v, c_off);
  }
}

// ------------------------------------------------------------------ TMA tiles
// A tile [BM x BK] of k-block k0 starting at row m0 into sa.
template <class C>
__device__ __forceinline__ void load_a(uint8_t* sa, const void* map, uint64_t* bar,
                                       const KParams& p, int k0, int m0) {
  if (!p.a_mn) {
    tma_load_2d(sa, map, bar, k0, m0);
  } else {
#pragma unroll
    for (int j = 0; j < BM / C::MN_ELEMS; ++j)
      tma_load_2d(sa + j * C::MN_CHUNK, map, bar, m0 + C::MN_ELEMS * j, k0);
  }
}

// This CTA's B rows of n-tile nt into sb. CG = 1: the whole [BN x BK] tile,
// two BN/2 halves (rows n0 and n0 + pair offset) for paired operands.
// CG = 2: CTA `rank` stages MMA columns [rank*BN/2, (rank+1)*BN/2), which
// for paired operands is the first (rank 0) or the paired (rank 1) half.
template <class C, int BN, int CG>
__device__ __forceinline__ void load_b(uint8_t* sb, const void* map, uint64_t* bar,
                                       const KParams& p, int k0, int nt, int rank) {
  constexpr int W = C::MN_ELEMS;
  if (CG == 2 || p.b_pair_off == 0) {
    const int n0 = p.b_pair_off == 0 ? nt * BN + rank * C::B_ROWS
                                     : nt * (BN / 2) + rank * p.b_pair_off;
    if (!p.b_mn) {
      tma_load_2d(sb, map, bar, k0, n0);
    } else {
#pragma unroll
      for (int j = 0; j < C::B_ROWS / W; ++j)
        tma_load_2d(sb + j * C::MN_CHUNK, map, bar, n0 + W * j, k0);
    }
  } else {
    const int n0 = nt * (BN / 2);
    if (!p.b_mn) {
      tma_load_2d(sb, map, bar, k0, n0);
      tma_load_2d(sb + (BN / 2) * C::ROW_BYTES, map, bar, k0, n0 + p.b_pair_off);
    } else {
#pragma unroll
      for (int j = 0; j < BN / 2 / W; ++j) {
        tma_load_2d(sb + j * C::MN_CHUNK, map, bar, n0 + W * j, k0);
        tma_load_2d(sb + (j + BN / 2 / W) * C::MN_CHUNK, map, bar, n0 + p.b_pair_off + W * j,
                    k0);
      }
    }
  }
}

// ------------------------------------------------------------------ kernel
// Persistent, warp-specialised. Units (tile, k-split) are strided over the
// CTAs (CG = 1) or over the CTA pairs of a 2-CTA cluster (CG = 2).
//
// CG = 2 hand-offs (even CTA = leader, the only one issuing MMAs):
//   producer (each CTA)  -> full[s]   own CTA   (TMA transaction bytes)
//   split warps (each)   -> split[s]  leader    (remote arrive, 2 x 8 warps)
//   leader MMA commit    -> empty[s]  both CTAs (tcgen05.commit multicast)
//   leader MMA commit    -> accf[b]   both CTAs (tcgen05.commit multicast)
//   epilogue warps (each)-> acce[b]   leader    (remote arrive, 2 x 4 warps)
// A cluster barrier after set-up (barrier init, TMEM alloc) and before
// teardown (TMEM dealloc, exit) keeps either CTA from touching the other's
// barriers or TMEM outside their lifetime.
// MODE 0: 3xTF32 (fp32-accurate). MODE 1: fp32 operands rounded to bf16 by
// the split warps (fp32 accumulate), one kind::f16 MMA per K-block. MODE 2:
// bf16 operands in global memory, staged by TMA as they are (64-deep
// K-blocks, SWIZZLE_128B) and fed to kind::f16 MMAs directly; the split
// warps have nothing to do and the MMA issuer waits on the TMA barrier.
template <int BN, int BK, int CG, int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC,
                       const __grid_constant__ CUtensorMap tmD, const KParams p) {
  rnet_dev::pdl_trigger();
  constexpr bool BF = MODE == 1;
  // MODE 2: four of the idle split warps (6-9) become a second epilogue set
  constexpr int NEPI = MODE == 2 ? 2 * NUM_EPI_WARPS : NUM_EPI_WARPS;
  constexpr int RELAY_WARP = FIRST_SPLIT_WARP + NUM_SPLIT_WARPS - 1;
  using C = Cfg<BN, BK, CG, MODE == 2 ? 2 : 4, MODE != 2, NEPI>;
  constexpr bool PAIR = CG == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* epi_tiles = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* split = bars + C::STAGES;
  uint64_t* empty = bars + 2 * C::STAGES;
  uint64_t* accf = bars + 3 * C::STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;
  const int group = PAIR ? blockIdx.x >> 1 : blockIdx.x;
  const int n_groups = PAIR ? gridDim.x >> 1 : gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split[s], MODE == 2 ? CG : NUM_SPLIT_WARPS * CG);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], NEPI * CG);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc<CG>(tmem_slot, C::TMEM_COLS);
    tmem_relinquish<CG>();
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  rnet_dev::pdl_wait();  // every global access below follows the preceding kernel

  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int unit = group; unit < p.num_units && ok; unit += n_groups) {
        int mt, nt0, nt1, kb0, kb1;
        unit_range(p, unit, mt, nt0, nt1, kb0, kb1);
        const int m0 = mt * BM * CG + rank * BM;
        for (int nt = nt0; nt < nt1 && ok; ++nt) {
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % C::STAGES;
            const uint32_t ph = (it / C::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, p.err, abort_flag)) { ok = false; break; }
            uint8_t* sa = smem + s * C::STAGE_BYTES;
            uint8_t* sb = sa + C::A_BYTES;
            mbar_arrive_expect_tx(&full[s], C::RAW_BYTES);
            const int k0 = kb * BK;
            load_a<C>(sa, &tmA, &full[s], p, k0, m0);
            load_b<C, BN, CG>(sb, &tmB, &full[s], p, k0, nt, rank);
          }
        }
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc(BM * CG, BN, 2, p.a_mn, p.b_mn);
      const uint32_t idesc_bf = make_idesc(BM * CG, BN, 1, 0, 0);  // bf16, both K-major
      const uint32_t idesc_st = make_idesc(BM * CG, BN, 1, p.a_mn, p.b_mn);  // MODE 2
      // Byte advance of one 8-deep K slice and LBO / SBO / layout per operand.
      const uint32_t a_kstep = p.a_mn ? 1024u : 32u;
      const uint32_t b_kstep = p.b_mn ? 1024u : 32u;
      const uint32_t a_lbo = p.a_mn ? (uint32_t)C::MN_CHUNK : 16u;
      const uint32_t b_lbo = p.b_mn ? (uint32_t)C::MN_CHUNK : 16u;
      const uint32_t a_sbo = p.a_mn ? 512u : C::K_SBO;
      const uint32_t b_sbo = p.b_mn ? 512u : C::K_SBO;
      const uint32_t a_lay = p.a_mn ? 1u : C::K_LAYOUT;
      const uint32_t b_lay = p.b_mn ? 1u : C::K_LAYOUT;
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int unit = group; unit < p.num_units && ok; unit += n_groups) {
        int mt, nt0, nt1, kb0, kb1;
        unit_range(p, unit, mt, nt0, nt1, kb0, kb1);
        for (int nt = nt0; nt < nt1 && ok; ++nt, ++tc) {
          const int ab = tc & 1;
          const uint32_t tph = (tc >> 1) & 1;
          if (!mbar_wait(&acce[ab], tph ^ 1, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tacc = tmem_base + ab * BN;
          uint32_t accumulate = 0;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % C::STAGES;
            const uint32_t ph = (it / C::STAGES) & 1;
            if (!mbar_wait((MODE == 2 && CG == 1) ? &full[s] : &split[s], ph, p.err,
                           abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(smem + s * C::STAGE_BYTES);
            if constexpr (MODE == 2) {
              // bf16 SWIZZLE_128B tiles: K-major rows of 64 elements (a
              // 16-deep slice is +32 B inside the swizzle atom; 8-row groups
              // 1024 B apart); MN-major: 64-wide MN chunks MN_CHUNK apart,
              // K rows 128 B apart (a 16-deep slice is +2048 B, 8-row K
              // groups 1024 B apart)
              const uint32_t b_hi = a_hi + C::A_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t da =
                    p.a_mn ? make_sdesc(a_hi + kk * 2048, C::MN_CHUNK, 1024, 2)
                           : make_sdesc(a_hi + kk * 32, 16, 1024, 2);
                const uint64_t db =
                    p.b_mn ? make_sdesc(b_hi + kk * 2048, C::MN_CHUNK, 1024, 2)
                           : make_sdesc(b_hi + kk * 32, 16, 1024, 2);
                umma_f16<CG>(tacc, da, db, idesc_st, accumulate);
                accumulate = 1;
              }
            } else if constexpr (BF) {
              // bf16 tiles (K-major, no swizzle) written by the split warps
              const uint32_t a_bf = a_hi + C::RAW_BYTES;
              const uint32_t b_bf = a_bf + BM * 32;
              umma_f16<CG>(tacc, make_sdesc(a_bf, 128, 256, 0), make_sdesc(b_bf, 128, 256, 0),
                           idesc_bf, accumulate);
              accumulate = 1;
            } else {
              const uint32_t b_hi = a_hi + C::A_BYTES;
              const uint32_t a_lo = a_hi + C::RAW_BYTES;
              const uint32_t b_lo = b_hi + C::RAW_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / 8; ++kk) {
                const uint64_t dah = make_sdesc(a_hi + kk * a_kstep, a_lbo, a_sbo, a_lay);
                const uint64_t dal = make_sdesc(a_lo + kk * a_kstep, a_lbo, a_sbo, a_lay);
                const uint64_t dbh = make_sdesc(b_hi + kk * b_kstep, b_lbo, b_sbo, b_lay);
                const uint64_t dbl = make_sdesc(b_lo + kk * b_kstep, b_lbo, b_sbo, b_lay);
                umma_tf32<CG>(tacc, dah, dbl, idesc, accumulate);
                umma_tf32<CG>(tacc, dal, dbh, idesc, 1);
                umma_tf32<CG>(tacc, dah, dbh, idesc, 1);
                accumulate = 1;
              }
            }
            if constexpr (PAIR) umma_commit_pair(&empty[s]); else umma_commit<CG>(&empty[s]);
          }
          if (!ok) break;
          if constexpr (PAIR) umma_commit_pair(&accf[ab]); else umma_commit<CG>(&accf[ab]);
        }
      }
      // Every issued MMA has finished before teardown releases TMEM (also on
      // the abort path, where no epilogue waited for the last ones).
      umma_commit<CG>(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, p.err, &no_abort);
    }
  } else if (warp >= FIRST_SPLIT_WARP && !(MODE == 2 && warp < FIRST_SPLIT_WARP + 4)) {
   if constexpr (MODE == 2 && CG == 2) {
    // bf16 tiles need no split work, but the pair's MMA (issued by the even
    // CTA) reads both CTAs' tiles: one thread per CTA relays "this CTA's
    // tiles of stage s have landed" to the even CTA's split[s] barrier
    if (warp == RELAY_WARP && lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int unit = group; unit < p.num_units && ok; unit += n_groups) {
        int mt, nt0, nt1, kb0, kb1;
        unit_range(p, unit, mt, nt0, nt1, kb0, kb1);
        for (int nt = nt0; nt < nt1 && ok; ++nt) {
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % C::STAGES;
            const uint32_t ph = (it / C::STAGES) & 1;
            if (!mbar_wait(&full[s], ph, p.err, abort_flag)) { ok = false; break; }
            mbar_arrive_cluster(&split[s], 0);
          }
        }
      }
    }
   } else if constexpr (MODE != 2) {
    const int t = threadIdx.x - FIRST_SPLIT_WARP * 32;
    constexpr int NT = NUM_SPLIT_WARPS * 32;
    constexpr int N4 = C::RAW_BYTES / 16;
    uint32_t it = 0;
    bool ok = true;
    for (int unit = group; unit < p.num_units && ok; unit += n_groups) {
      int mt, nt0, nt1, kb0, kb1;
      unit_range(p, unit, mt, nt0, nt1, kb0, kb1);
      for (int nt = nt0; nt < nt1 && ok; ++nt) {
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.err, abort_flag)) { ok = false; break; }
          if constexpr (BF) {
            // Round the raw fp32 tiles (unswizzled: K-major [rows][16], MN-major
            // 32-wide chunks of [16 k-rows][32]) to bf16 into K-major core-matrix
            // order: row r, K-chunk c (8 values) at (r/8)*256 + c*128 + (r%8)*16.
            // A warp handles 32 consecutive rows of one K-chunk.
            const uint8_t* rawb = smem + s * C::STAGE_BYTES;
            uint8_t* bfb = smem + s * C::STAGE_BYTES + C::RAW_BYTES;
            constexpr int ROWS_ALL = BM + C::B_ROWS;
#pragma unroll 2
            for (int q = t; q < 2 * ROWS_ALL; q += NT) {
              const int kc = (q >> 5) & 1;
              const int r = (q & 31) + 32 * (q >> 6);
              const bool is_a = r < BM;
              const int rr = is_a ? r : r - BM;
              const uint8_t* src = rawb + (is_a ? 0 : C::A_BYTES);
              float v[8];
              if (!(is_a ? p.a_mn : p.b_mn)) {
                const float4* s4 = reinterpret_cast<const float4*>(src + rr * 64 + kc * 32);
                const float4 x0 = s4[0], x1 = s4[1];
                v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
                v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
              } else {
                const float* sf =
                    reinterpret_cast<const float*>(src + (rr >> 5) * C::MN_CHUNK + (rr & 31) * 4);
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = sf[(kc * 8 + u) * 32];
              }
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                w[i] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i])) |
                       ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * i + 1])) << 16);
              *reinterpret_cast<uint4*>(bfb + (is_a ? 0 : BM * 32) + (rr >> 3) * 256 + kc * 128 +
                                        (rr & 7) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
            const float4* raw = reinterpret_cast<const float4*>(smem + s * C::STAGE_BYTES);
            float4* lo = reinterpret_cast<float4*>(smem + s * C::STAGE_BYTES + C::RAW_BYTES);
            // lo = x - (x with the low 13 mantissa bits cleared); the layout is
            // elementwise-identical to the raw tile, so swizzling is irrelevant
#pragma unroll 4
            for (int i = t; i < N4; i += NT) {
              const float4 x = raw[i];
              float4 l;
              l.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
              l.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
              l.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
              l.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
              lo[i] = l;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) mbar_arrive_cluster(&split[s], 0); else mbar_arrive(&split[s]);
          }
        }
      }
    }
   }
  } else {  // epilogue warps 0..3 (+ 6..9 in MODE 2)
    const int q = warp & 3;  // TMEM lane quadrant (warp i may access lanes 32 (i % 4) + ...)
    const int eset = warp < NUM_EPI_WARPS ? 0 : 1;
    const int eslot = eset * NUM_EPI_WARPS + q;
    uint32_t tc = 0;
    bool ok = true;
    for (int unit = group; unit < p.num_units && ok; unit += n_groups) {
      int mt, nt0, nt1, kb0, kb1;
      unit_range(p, unit, mt, nt0, nt1, kb0, kb1);
      const int row0 = mt * BM * CG + rank * BM + q * 32;
      Top2State st{-1e30f, -1e30f, 0, 0};
      for (int nt = nt0; nt < nt1; ++nt, ++tc) {
        const int ab = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        prefetch_epilogue_inputs<BN>(p, row0 + lane, nt);
        if (!mbar_wait(&accf[ab], tph, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tacc = tmem_base + ((uint32_t)(q * 32) << 16) + ab * BN;
        const size_t c_off =
            p.split_stride ? (size_t)p.split_stride * (size_t)(kb0 / p.kb_per_split) : 0;
        epilogue_subtile<BN, MODE != 2>(p, tacc, row0, nt, nt == nt1 - 1, st,
                             epi_tiles + eslot * EPI_TILE_FLOATS, c_off, eset,
                             NEPI / NUM_EPI_WARPS, &tmC, &tmD);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) mbar_arrive_cluster(&acce[ab], 0); else mbar_arrive(&acce[ab]);
        }
      }
    }
    // the warp's bulk stores have completed before the CTA exits
    if ((p.tma_out || p.swiglu_planes) && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc<CG>(tmem_base, C::TMEM_COLS);
}

// ------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D fp32 (or bf16) tensor map. box = {box_inner, box_outer} elements.
static bool make_map(CUtensorMap* m, const float* base, uint64_t inner, uint64_t outer,
                     uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swz, bool bf16 = false) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * (bf16 ? 2 : 4)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<float*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_map_f32(CUtensorMap* m, const float* base, int rank, const uint64_t* dims,
                    const uint64_t* stride_bytes, const uint32_t* box) {
  auto enc = get_encode_fn();
  if (!enc || rank < 1 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = stride_bytes[i];
  }
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float*>(base), d, st, bx,
                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Which argument check or launch step failed last (thread-local).
static thread_local const char* g_reason = "";
const char* gemm_last_reason() { return g_reason; }
static cudaError_t reject(const char* why) {
  g_reason = why;
  return cudaErrorInvalidValue;
}

// Test hook: force the CTA group (0 = automatic).
static int g_force_cg = 0;
// RNET_GEMM_TMA_OUT=0 keeps the bf16 path's stores on the warps (A/B timing)
static const bool g_tma_out = [] {
  const char* e = getenv("RNET_GEMM_TMA_OUT");
  return !(e && e[0] == '0');
}();
void set_force_cta_group(int cg) { g_force_cg = (cg == 1 || cg == 2) ? cg : 0; }

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, int BK, int CG, int MODE>
static cudaError_t launch(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tb,
                          const CUtensorMap& tc, const CUtensorMap& td, const KParams& kp) {
  using C = Cfg<BN, BK, CG, MODE == 2 ? 2 : 4, MODE != 2,
                MODE == 2 ? 2 * NUM_EPI_WARPS : NUM_EPI_WARPS>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, BK, CG, MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) {
      g_reason = "shared-memory attribute";
      return e;
    }
    configured = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CG;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  // RNET_GEMM_PDL=0 launches without programmatic serialization (A/B timing).
  static const bool pdl = [] {
    const char* e = getenv("RNET_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  cfg.attrs = pdl ? attr : attr + 1;
  cfg.numAttrs = (CG > 1 ? 1 : 0) + (pdl ? 1 : 0);
  // Persistent grid: one CTA (pair) per SM (pair) that can be co-resident.
  static int max_groups = 0;
  if (max_groups == 0) {
    max_groups = num_sms() / CG;
    if (CG > 1) {
      int n = 0;
      cfg.gridDim = dim3(max_groups * CG);
      if (cudaOccupancyMaxActiveClusters(&n, gemm_tf32x3_kernel<BN, BK, CG, MODE>, &cfg) ==
              cudaSuccess &&
          n > 0 && n < max_groups)
        max_groups = n;
      cudaGetLastError();
    }
    if (getenv("RNET_GEMM_VERBOSE"))
      fprintf(stderr, "gemm_tf32x3<BN=%d, CG=%d>: %d co-resident CTA groups, %d stages, %d B smem\n",
              BN, CG, max_groups, C::STAGES, C::SMEM_BYTES);
  }
  const int groups = kp.num_units < max_groups ? kp.num_units : max_groups;
  cfg.gridDim = dim3(groups * CG);
  cudaError_t e =
      cudaLaunchKernelEx(&cfg, gemm_tf32x3_kernel<BN, BK, CG, MODE>, ta, tb, tc, td, kp);
  if (e != cudaSuccess) {
    g_reason = "kernel launch";
    return e;
  }
  return rnet_k::launched();
}

// ------------------------------------------------------------------ split-K workspace
// Short-M GEMMs (decode steps, small batches) have too few output tiles to
// fill the GPU. Their K range is split over extra CTAs that store partial
// tiles into a workspace; splitk_reduce sums the partials in split order (so
// results do not depend on scheduling) and applies the epilogue.
// Paired-column rules over S partial planes [M, 2h] (S = 1: a stored C):
// a = sum of column f, b = sum of column h + f, summed in split order.
// Same formulas (sigmoid_fast / silu_fast) as the training forward's SwiGLU
// epilogue and MinGRU scan.
__global__ void __launch_bounds__(256)
    splitk_pair_kernel(const float* __restrict__ ws, int S, int M, int h, Epilogue e) {
  rnet_dev::pdl_trigger();
  const size_t plane = (size_t)M * 2 * h;
  const int h4 = h >> 2;
  const size_t n4 = (size_t)M * h4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / h4;
    const int c = (int)(i - r * h4) * 4;
    const float* src = ws + r * 2 * h + c;
    float4 a = *reinterpret_cast<const float4*>(src);
    float4 b = *reinterpret_cast<const float4*>(src + h);
    for (int k = 1; k < S; ++k) {
      const float4 pa = *reinterpret_cast<const float4*>(src + k * plane);
      const float4 pb = *reinterpret_cast<const float4*>(src + k * plane + h);
      a.x += pa.x; a.y += pa.y; a.z += pa.z; a.w += pa.w;
      b.x += pb.x; b.y += pb.y; b.z += pb.z; b.w += pb.w;
    }
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    const size_t o = r * e.ldf + c;
    if (e.kind == EPI_PAIR_SILU) {
#pragma unroll
      for (int j = 0; j < 4; ++j) e.H[o + j] = silu_fast(av[j]) * bv[j];
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float z = sigmoid_fast(av[j] + e.b0[c + j]);
        const float ht = bv[j] + e.b1[c + j];
        const float hn = (1.f - z) * e.state[o + j] + z * ht;
        e.state[o + j] = hn;
        e.xres[o + j] += hn;
      }
    }
  }
}

__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ ws, int S, int M, int N, Epilogue e) {
  rnet_dev::pdl_trigger();
  const size_t plane = (size_t)M * N;
  if ((N & 3) == 0) {
    const int N4 = N >> 2;
    const size_t n4 = (size_t)M * N4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
      const size_t r = i / N4;
      const int c = (int)(i - r * N4) * 4;
      const float* src = ws + r * N + c;
      float4 a = *reinterpret_cast<const float4*>(src);
      // loads in batches of 8 (independent), additions in split order
      for (int k0 = 1; k0 < S; k0 += 8) {
        float4 b[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < S) b[j] = *reinterpret_cast<const float4*>(src + (k0 + j) * plane);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < S) { a.x += b[j].x; a.y += b[j].y; a.z += b[j].z; a.w += b[j].w; }
      }
      float* dst = e.C + r * e.ldc + c;
      const float al = e.alpha;
      float4 o = make_float4(al * a.x, al * a.y, al * a.z, al * a.w);
      if (e.kind == EPI_ACCUM || e.kind == EPI_RESID) {
        const float* base = e.kind == EPI_ACCUM ? dst : e.R + r * e.ldr + c;
        o.x += base[0]; o.y += base[1]; o.z += base[2]; o.w += base[3];
      }
      dst[0] = o.x; dst[1] = o.y; dst[2] = o.z; dst[3] = o.w;
    }
  } else {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < plane;
         i += (size_t)gridDim.x * blockDim.x) {
      const size_t r = i / N;
      const int c = (int)(i - r * N);
      float a = ws[i];
      for (int k = 1; k < S; ++k) a += ws[i + k * plane];
      float* dst = e.C + r * e.ldc + c;
      float o = e.alpha * a;
      if (e.kind == EPI_ACCUM) o += *dst;
      if (e.kind == EPI_RESID) o += e.R[r * e.ldr + c];
      *dst = o;
    }
  }
}

// Row-owner forms of the two sums above, for epilogues that also normalise
// the finished rows (Epilogue::ny): one CTA per row, threads owning columns
// c = 4 * tid + 4 * blockDim.x * j. Pass 1 sums in split order, applies the
// epilogue, stores the row and accumulates its sum of squares; pass 2
// re-reads the thread's own stores and writes y = x * rsqrt(ms + eps) * w
// (the RMSNorm forward's formula). S = 0: the GEMM stored the row already.
__device__ __forceinline__ float block_sum_128(float v, float* red) {
  v = rnet_dev::warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const float t = red[0] + red[1] + red[2] + red[3];
  return t;
}

__device__ __forceinline__ void norm_row_pass(const float* x, const float* w, float* y, int n,
                                              float ri) {
  for (int c = threadIdx.x * 4; c < n; c += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + c);
    const float4 g = *reinterpret_cast<const float4*>(w + c);
    *reinterpret_cast<float4*>(y + c) =
        make_float4(v.x * ri * g.x, v.y * ri * g.y, v.z * ri * g.z, v.w * ri * g.w);
  }
}

constexpr int NORM_THREADS = 128;

__global__ void __launch_bounds__(NORM_THREADS)
    splitk_reduce_norm_kernel(const float* __restrict__ ws, int S, int M, int N, Epilogue e) {
  rnet_dev::pdl_trigger();
  __shared__ float red[NORM_THREADS / 32];
  const size_t r = blockIdx.x;
  const size_t plane = (size_t)M * N;
  float* dst = e.C + r * e.ldc;
  float ss = 0.f;
  for (int c = threadIdx.x * 4; c < N; c += blockDim.x * 4) {
    float4 o;
    if (S > 0) {
      const float* src = ws + r * N + c;
      float4 a = *reinterpret_cast<const float4*>(src);
      for (int k0 = 1; k0 < S; k0 += 8) {
        float4 b[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < S) b[j] = *reinterpret_cast<const float4*>(src + (k0 + j) * plane);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < S) { a.x += b[j].x; a.y += b[j].y; a.z += b[j].z; a.w += b[j].w; }
      }
      const float al = e.alpha;
      o = make_float4(al * a.x, al * a.y, al * a.z, al * a.w);
      if (e.kind == EPI_ACCUM || e.kind == EPI_RESID) {
        const float* base = e.kind == EPI_ACCUM ? dst + c : e.R + r * e.ldr + c;
        o.x += base[0]; o.y += base[1]; o.z += base[2]; o.w += base[3];
      }
      *reinterpret_cast<float4*>(dst + c) = o;
    } else {
      o = *reinterpret_cast<const float4*>(dst + c);
    }
    ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
  }
  ss = block_sum_128(ss, red);
  const float ri = rsqrtf(ss / (float)N + e.eps);
  if (!e.conv_out) {
    norm_row_pass(dst, e.nw, e.ny + r * e.ldc, N, ri);
    return;
  }
  const int pos = *e.pos;
  float* ring_row = e.ring + r * rnet_dev::CONV_RING * N;
  for (int c = threadIdx.x * 4; c < N; c += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(dst + c);
    const float4 g = *reinterpret_cast<const float4*>(e.nw + c);
    const float4 y = make_float4(v.x * ri * g.x, v.y * ri * g.y, v.z * ri * g.z, v.w * ri * g.w);
    *reinterpret_cast<float4*>(e.ny + r * e.ldc + c) = y;
    *reinterpret_cast<float4*>(e.conv_out + r * N + c) =
        rnet_dev::conv_step4(y, ring_row, pos, e.cw3, e.cw7, e.cw15, c, N);
  }
}

// EPI_PAIR_GRU with the norm: the same update as splitk_pair_kernel, then the
// RMSNorm of the updated residual row.
__global__ void __launch_bounds__(NORM_THREADS)
    splitk_pair_gru_norm_kernel(const float* __restrict__ ws, int S, int M, int h, Epilogue e) {
  rnet_dev::pdl_trigger();
  __shared__ float red[NORM_THREADS / 32];
  const size_t r = blockIdx.x;
  const size_t plane = (size_t)M * 2 * h;
  float ss = 0.f;
  for (int c = threadIdx.x * 4; c < h; c += blockDim.x * 4) {
    const float* src = ws + r * 2 * h + c;
    float4 a = *reinterpret_cast<const float4*>(src);
    float4 b = *reinterpret_cast<const float4*>(src + h);
    for (int k = 1; k < S; ++k) {
      const float4 pa = *reinterpret_cast<const float4*>(src + k * plane);
      const float4 pb = *reinterpret_cast<const float4*>(src + k * plane + h);
      a.x += pa.x; a.y += pa.y; a.z += pa.z; a.w += pa.w;
      b.x += pb.x; b.y += pb.y; b.z += pb.z; b.w += pb.w;
    }
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    const size_t o = r * e.ldf + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float z = sigmoid_fast(av[j] + e.b0[c + j]);
      const float ht = bv[j] + e.b1[c + j];
      const float hn = (1.f - z) * e.state[o + j] + z * ht;
      e.state[o + j] = hn;
      const float xn = e.xres[o + j] + hn;
      e.xres[o + j] = xn;
      ss += xn * xn;
    }
  }
  ss = block_sum_128(ss, red);
  const float ri = rsqrtf(ss / (float)h + e.eps);
  norm_row_pass(e.xres + r * e.ldf, e.nw, e.ny + r * e.ldf, h, ri);
}

struct Workspace {
  float* p = nullptr;
  size_t floats = 0;
};
static std::mutex g_ws_mu;
// one workspace per (device, stream): GEMMs on one stream are ordered
static std::vector<std::pair<std::pair<int, cudaStream_t>, Workspace>> g_ws;

static Workspace* workspace_for(cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_ws_mu);
  for (auto& e : g_ws)
    if (e.first.first == dev && e.first.second == s) return &e.second;
  g_ws.push_back({{dev, s}, Workspace{}});
  return &g_ws.back().second;
}

cudaError_t reserve_workspace(cudaStream_t stream, size_t floats) {
  Workspace* w = workspace_for(stream);
  if (w->floats >= floats) return cudaSuccess;
  if (w->p) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    cudaFree(w->p);
    w->p = nullptr;
    w->floats = 0;
  }
  cudaError_t e = cudaMalloc(&w->p, floats * sizeof(float));
  if (e != cudaSuccess) {
    w->p = nullptr;
    return e;
  }
  w->floats = floats;
  return cudaSuccess;
}

cudaError_t gemm_tf32x3(cudaStream_t stream, int M, int N, int K, const Operand& A,
                        const Operand& B, const Epilogue& epi_in, int b_pair_off, int k_splits,
                        unsigned* err_word, int precision) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  g_reason = "";
  // paired-column epilogues: the GEMM itself stores (into the workspace
  // planes or C), the pair rule runs where the result is read back
  const bool pair = epi_in.kind == EPI_PAIR_SILU || epi_in.kind == EPI_PAIR_GRU;
  if (pair && (N != 2 * epi_in.ldf || epi_in.ldf % 4 || b_pair_off || epi_in.C == nullptr))
    return reject("paired epilogue: N must be 2 * ldf (ldf % 4 == 0) with C as scratch");
  const bool norm = epi_in.ny != nullptr;
  if (norm) {
    const bool ok_kind = epi_in.kind == EPI_PAIR_GRU || epi_in.kind == EPI_STORE ||
                         epi_in.kind == EPI_ACCUM || epi_in.kind == EPI_RESID;
    const int width = pair ? epi_in.ldf : N;
    const int pitch = pair ? epi_in.ldf : epi_in.ldc;
    if (!ok_kind || !epi_in.nw || width % 4 || pitch % 4 || epi_in.C16 || b_pair_off ||
        epi_in.splits_out ||
        (epi_in.conv_out && (pair || !epi_in.ring || !epi_in.pos || !epi_in.cw3 ||
                             !epi_in.cw7 || !epi_in.cw15)))
      return reject("row norm: store / residual / GRU-pair epilogue, width % 4 == 0, weights");
  }
  if (epi_in.splits_out && (epi_in.kind != EPI_STORE || !epi_in.planes_out ||
                            epi_in.ldc != N || epi_in.C16 || b_pair_off))
    return reject("deferred split-K sum: EPI_STORE with ldc == N and both outputs");
  Epilogue epi = epi_in;
  epi.ny = nullptr;  // the GEMM kernel itself never normalises
  epi.splits_out = nullptr;
  epi.planes_out = nullptr;
  if (pair) {
    epi.kind = EPI_STORE;
    epi.ldc = N;
    epi.alpha = 1.0f;
  }
  if (K <= 0 || A.p == nullptr || B.p == nullptr) return reject("K <= 0 or null operand");
  if (A.bf16 != B.bf16) return reject("one bf16 and one fp32 operand");
  const bool st16 = A.bf16;  // bf16 storage: MODE 2
  const bool bf = !st16 && precision == PREC_BF16;
  const int ld_mult = st16 ? 8 : 4;
  if ((A.ld % ld_mult) || (B.ld % ld_mult) || (reinterpret_cast<uintptr_t>(A.p) & 15) ||
      (reinterpret_cast<uintptr_t>(B.p) & 15))
    return reject("operand row pitch not a multiple of 16 bytes or operand not 16-byte aligned");
  if (st16 && (b_pair_off % 8)) return reject("bf16 paired offset not a multiple of 8");
  const bool paired = b_pair_off > 0;
  const bool row_owner = epi.kind == EPI_TOP2;
  const int BK = st16 ? 64 : 16;
  // Short M: split K over a workspace when the output tiles cannot fill the
  // SMs (store / residual epilogues, and accumulation asked for in one pass).
  int ws_splits = 1;
  if (!paired && !row_owner && g_force_cg == 0 && M <= 1024 && !epi.C16 &&
      (epi.kind == EPI_STORE || epi.kind == EPI_RESID ||
       (epi.kind == EPI_ACCUM && k_splits == 1))) {
    const int tiles = ((M + BM - 1) / BM) * ((N + 127) / 128);
    const int kb = (K + BK - 1) / BK;
    int sp = num_sms() / tiles;
    if (sp > kb / 2) sp = kb / 2;  // >= 2 k-blocks per split
    static const int sp_max = [] {
      const char* v = getenv("RNET_SPLITK_MAX");
      return v && atoi(v) >= 2 ? atoi(v) : 32;
    }();
    if (sp > sp_max) sp = sp_max;
    if (sp >= 2) {
      const size_t need = (size_t)sp * M * N;
      Workspace* w = workspace_for(stream);
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(stream, &cs);
      if (w->floats < need && cs == cudaStreamCaptureStatusNone)
        reserve_workspace(stream, need);  // on failure: no split
      if (w->floats >= need) ws_splits = sp;
    }
  }
  // CTA pairs (one 256-row MMA over two SMs, each staging half of B) cut
  // shared-memory and L2->SM traffic per FLOP by a third; single CTAs are kept
  // for short M, where pairs would leave SMs idle.
  const int CG = g_force_cg > 0 ? g_force_cg : (M > BM && ws_splits == 1 ? 2 : 1);
  // CG = 1: paired-B and row-owner epilogues use 128-wide tiles (64-feature
  // halves). CG = 2: 256-wide tiles (each CTA stages one 128-row half).
  // (16-deep K-blocks, 4-6 stages, measured 5-20% faster than 32-deep.)
  const int BN = CG == 2 ? (N <= 128 && !paired ? 128 : 256)
                         : ((paired || row_owner || N <= 128 || ws_splits > 1) ? 128 : 256);
  const int n_logical_tile = paired ? BN / 2 : BN;

  KParams kp{};
  kp.M = M;
  kp.N = N;
  kp.K = K;
  kp.m_tiles = (M + BM * CG - 1) / (BM * CG);
  kp.n_tiles = (N + n_logical_tile - 1) / n_logical_tile;
  kp.kb_total = (K + BK - 1) / BK;
  kp.row_owner = row_owner ? 1 : 0;
  kp.b_pair_off = b_pair_off;
  kp.a_mn = A.mn_major ? 1 : 0;
  kp.b_mn = B.mn_major ? 1 : 0;
  kp.epi = epi;
  kp.err = err_word;
  kp.stage_epi = st16 ? 1 : 0;  // fp32 tiles: set below when TMA can store

  int splits = 1;
  if (ws_splits > 1) {
    splits = ws_splits;
    Epilogue part;  // partial tiles: plain stores into the workspace
    part.kind = EPI_STORE;
    part.C = workspace_for(stream)->p;
    part.ldc = N;
    kp.epi = part;
    kp.split_stride = (long long)M * N;
  } else if (epi.kind == EPI_ACCUM) {
    if (k_splits > 0) {
      splits = k_splits;
    } else {
      const int tiles = kp.m_tiles * kp.n_tiles;
      const int groups = num_sms() / CG;
      if (tiles < groups) splits = groups / tiles;
      // keep each split's K at most 2048 so the TMEM accumulation stays
      // fp32-accurate, and at least 4 k-blocks so a split is worth a tile
      const int min_splits = (K + 2047) / 2048;
      if (splits < min_splits) splits = min_splits;
      const int max_splits = kp.kb_total / 4 > 0 ? kp.kb_total / 4 : 1;
      if (splits > max_splits) splits = max_splits;
    }
  }
  if (splits < 1) splits = 1;
  kp.kb_per_split = (kp.kb_total + splits - 1) / splits;
  kp.k_splits = (kp.kb_total + kp.kb_per_split - 1) / kp.kb_per_split;
  kp.num_units = row_owner ? kp.m_tiles : kp.m_tiles * kp.n_tiles * kp.k_splits;

  // bf16 (MODE 1): the split warps read the raw fp32 tiles, so they stay
  // unswizzled. bf16 storage (MODE 2): 128-byte rows, SWIZZLE_128B both ways.
  const CUtensorMapSwizzle kswz =
      st16 ? CU_TENSOR_MAP_SWIZZLE_128B
           : bf ? CU_TENSOR_MAP_SWIZZLE_NONE
                : (BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  const CUtensorMapSwizzle mswz =
      st16 ? CU_TENSOR_MAP_SWIZZLE_128B
           : bf ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const uint32_t mn_box = st16 ? 64 : 32;
  auto map_a = [&](CUtensorMap* m, const float* base) {
    return !A.mn_major ? make_map(m, base, (uint64_t)K, (uint64_t)M, A.ld, BK, BM, kswz, st16)
                       : make_map(m, base, (uint64_t)M, (uint64_t)K, A.ld, mn_box, BK, mswz, st16);
  };
  const uint64_t b_rows = paired ? (uint64_t)b_pair_off + N : (uint64_t)N;
  // K-major box rows = the rows one TMA copy stages (a half tile when paired
  // or when a CTA pair splits B).
  const uint32_t b_box = (paired || CG == 2) ? BN / 2 : BN;
  auto map_b = [&](CUtensorMap* m, const float* base) {
    return !B.mn_major ? make_map(m, base, (uint64_t)K, b_rows, B.ld, BK, b_box, kswz, st16)
                       : make_map(m, base, b_rows, (uint64_t)K, B.ld, mn_box, BK, mswz, st16);
  };
  CUtensorMap ta, tb, tc, td;
  std::memset(&td, 0, sizeof(td));
  if (!map_a(&ta, A.p)) return reject("tensor map of A rejected");
  if (!map_b(&tb, B.p)) return reject("tensor map of B rejected");
  // plain stores / accumulations leave through TMA when C allows a tensor
  // map (16-byte aligned base and row pitch); otherwise the warps store the
  // tile through shared memory as coalesced rows
  std::memset(&tc, 0, sizeof(tc));
  kp.tma_out = 0;
  kp.copy16_tma = 0;
  // a store's bf16 copy leaves through TMA too when its map can be made
  if (kp.split_stride == 0 && g_tma_out && epi.kind == EPI_STORE && epi.C16 &&
      epi.ldc % 8 == 0 && (reinterpret_cast<uintptr_t>(epi.C16) & 15) == 0 &&
      make_map(&td, reinterpret_cast<const float*>(epi.C16), (uint64_t)N, (uint64_t)M, epi.ldc,
               32, 32, CU_TENSOR_MAP_SWIZZLE_NONE, true))
    kp.copy16_tma = 1;
  if (kp.split_stride == 0 && g_tma_out &&
      ((epi.kind == EPI_STORE && (epi.C16 == nullptr || kp.copy16_tma)) ||
       epi.kind == EPI_ACCUM) &&
      (reinterpret_cast<uintptr_t>(epi.C) & 15) == 0 &&
      epi.ldc % 4 == 0 && epi.ldc >= N &&
      make_map(&tc, epi.C, (uint64_t)N, (uint64_t)M, epi.ldc, 32, 32,
               CU_TENSOR_MAP_SWIZZLE_128B))
    kp.tma_out = 1;
  // split-K partial planes: one 3-D map over the workspace, z = split index
  if (kp.split_stride != 0 && g_tma_out && N % 4 == 0) {
    auto enc = get_encode_fn();
    cuuint64_t d[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)kp.k_splits};
    cuuint64_t st[2] = {(cuuint64_t)N * 4, (cuuint64_t)M * N * 4};
    cuuint32_t bx[3] = {32, 32, 1}, es[3] = {1, 1, 1};
    if (enc && enc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, kp.epi.C, d, st, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      kp.tma_out = 2;
  }
  // SwiGLU forward: G, U (and H) through one 3-D map when they are
  // equally spaced planes (the engine allocates them back to back)
  kp.swiglu_planes = 0;
  if (epi.kind == EPI_SWIGLU_FWD && kp.split_stride == 0 && g_tma_out && epi.G && epi.U &&
      epi.U > epi.G && epi.ldf % 4 == 0 && epi.ldf >= N &&
      ((reinterpret_cast<uintptr_t>(epi.G) & 15) == 0)) {
    const size_t plane = (size_t)(epi.U - epi.G);
    const bool h_adj = epi.H && epi.H16 == nullptr && (size_t)(epi.H - epi.U) == plane;
    const int planes = h_adj ? 3 : 2;
    if (plane % 4 == 0 && plane >= (size_t)M * epi.ldf) {
      const uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)planes};
      const uint64_t strides[2] = {(uint64_t)epi.ldf * 4, (uint64_t)plane * 4};
      const uint32_t box[3] = {32, 32, 1};
      auto enc = get_encode_fn();
      cuuint64_t d[3] = {dims[0], dims[1], dims[2]}, st[2] = {strides[0], strides[1]};
      cuuint32_t bx[3] = {box[0], box[1], box[2]}, es[3] = {1, 1, 1};
      if (enc &&
          enc(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(epi.G), d, st, bx, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
        kp.swiglu_planes = planes;
    }
  }
  if (kp.swiglu_planes == 2 && epi.H16 && epi.H == nullptr && epi.ldf % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(epi.H16) & 15) == 0 &&
      make_map(&td, reinterpret_cast<const float*>(epi.H16), (uint64_t)N, (uint64_t)M, epi.ldf,
               32, 32, CU_TENSOR_MAP_SWIZZLE_NONE, true))
    kp.copy16_tma = 1;
  // fp32 tiles: the staged path only pays with TMA stores (split-K partial
  // planes and residual epilogues keep thread-per-row stores, which leave
  // shared memory to the split warps)
  if (kp.tma_out) kp.stage_epi = 1;

  cudaError_t e;
  if (st16) {
    if (CG == 2)
      e = BN == 128 ? launch<128, 64, 2, 2>(stream, ta, tb, tc, td, kp)
                    : launch<256, 64, 2, 2>(stream, ta, tb, tc, td, kp);
    else
      e = BN == 128 ? launch<128, 64, 1, 2>(stream, ta, tb, tc, td, kp)
                    : launch<256, 64, 1, 2>(stream, ta, tb, tc, td, kp);
  } else if (bf) {
    if (CG == 2)
      e = BN == 128 ? launch<128, 16, 2, 1>(stream, ta, tb, tc, td, kp)
                    : launch<256, 16, 2, 1>(stream, ta, tb, tc, td, kp);
    else
      e = BN == 128 ? launch<128, 16, 1, 1>(stream, ta, tb, tc, td, kp)
                    : launch<256, 16, 1, 1>(stream, ta, tb, tc, td, kp);
  } else {
    if (CG == 2)
      e = BN == 128 ? launch<128, 16, 2, 0>(stream, ta, tb, tc, td, kp)
                    : launch<256, 16, 2, 0>(stream, ta, tb, tc, td, kp);
    else
      e = BN == 128 ? launch<128, 16, 1, 0>(stream, ta, tb, tc, td, kp)
                    : launch<256, 16, 1, 0>(stream, ta, tb, tc, td, kp);
  }
  if (e != cudaSuccess) return e;
  if (pair) {
    // fixed-order sum of the partials (or the stored C) + the pair rule
    const float* src = kp.split_stride ? kp.epi.C : epi.C;
    const int S = kp.split_stride ? kp.k_splits : 1;
    const size_t work = (size_t)M * (N / 2) / 4;
    size_t grid = (work + 255) / 256;
    if (grid > (size_t)num_sms() * 8) grid = (size_t)num_sms() * 8;
    if (grid < 1) grid = 1;
    if (norm)
      splitk_pair_gru_norm_kernel<<<(unsigned)M, NORM_THREADS, 0, stream>>>(src, S, M, N / 2,
                                                                            epi_in);
    else
      splitk_pair_kernel<<<(unsigned)grid, 256, 0, stream>>>(src, S, M, N / 2, epi_in);
    return rnet_k::launched();
  }
  if (epi_in.splits_out) {
    // the caller's kernel sums the planes (or reads C when unsplit)
    *epi_in.splits_out = kp.split_stride ? kp.k_splits : 1;
    *epi_in.planes_out = kp.split_stride ? kp.epi.C : epi_in.C;
    return e;
  }
  if (norm) {
    // fixed-order sum (none when unsplit) + epilogue + RMSNorm, a CTA per row
    const int S = kp.split_stride ? kp.k_splits : 0;
    splitk_reduce_norm_kernel<<<(unsigned)M, NORM_THREADS, 0, stream>>>(kp.epi.C, S, M, N,
                                                                        epi_in);
    return rnet_k::launched();
  }
  if (kp.split_stride == 0) return e;
  // fixed-order sum of the partials + the caller's epilogue
  const size_t work = (N % 4 == 0) ? (size_t)M * N / 4 : (size_t)M * N;
  size_t grid = (work + 255) / 256;
  if (grid > (size_t)num_sms() * 8) grid = (size_t)num_sms() * 8;
  splitk_reduce_kernel<<<(unsigned)grid, 256, 0, stream>>>(kp.epi.C, kp.k_splits, M, N, epi);
  return rnet_k::launched();
}

}  // namespace rnet_gemm
