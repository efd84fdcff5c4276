// Host-side interface of the tcgen05 GEMM engine (3xTF32 split, fp32 in/out).
//
//   C[M,N] (epilogue)= A[M,K] * B[N,K]^T
//
// Each operand is either K-major (element (i,k) at p[i*ld + k]) or MN-major
// (element (i,k) at p[k*ld + i]); both are consumed natively by TMA + UMMA
// (kind::tf32 supports MN-major operands on sm_100a).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rnet_gemm {

struct Operand {
  const float* p = nullptr;  // fp32 data, or bf16 data when bf16 is set
  int ld = 0;            // elements between consecutive stored rows
  bool mn_major = false; // see header comment
  bool bf16 = false;     // bf16 elements (both operands must then be bf16)
};

// A bf16 operand (ld a multiple of 8, base 16-byte aligned).
inline Operand bf16_operand(const __nv_bfloat16* p, int ld, bool mn_major) {
  Operand o;
  o.p = reinterpret_cast<const float*>(p);
  o.ld = ld;
  o.mn_major = mn_major;
  o.bf16 = true;
  return o;
}

enum EpiKind : int {
  EPI_STORE = 0,       // C = alpha*acc
  EPI_ACCUM = 1,       // C += alpha*acc        (vector red.add; split-K safe)
  EPI_RESID = 2,       // C = R + alpha*acc
  EPI_SWIGLU_FWD = 3,  // paired B: G = acc[gate], U = acc[up], H = silu(G)*U
  EPI_TOP2 = 5,        // row-owner: running top-2 over N, softmax, idx/w (+optional C)
  // Paired-column epilogues of a plain GEMM whose N = 2 * ldf columns are
  // two halves [a | b]; applied where the split-K partials are summed (no
  // extra launch), or after a plain store into C when K is not split.
  EPI_PAIR_SILU = 6,   // H[r, f] = silu(a) * b          (C: [M, 2 ldf] scratch)
  EPI_PAIR_GRU = 7,    // z = sigmoid(a + b0), h~ = b + b1, state = (1 - z) state + z h~,
                       // xres += state                  (state, xres: [M, ldf])
};

struct Epilogue {
  int kind = EPI_STORE;
  float alpha = 1.0f;
  float* C = nullptr;
  int ldc = 0;
  const float* R = nullptr;  // residual (EPI_RESID)
  int ldr = 0;
  // SwiGLU forward: gate / up pre-activations and hidden output, all [M, ldf]
  float* G = nullptr;
  float* U = nullptr;
  float* H = nullptr;
  int ldf = 0;
  // top-2
  int* topk_idx = nullptr;
  float* topk_w = nullptr;
  // optional bf16 copies of the stored result (row stride ldc for C16, ldf
  // for H16), for a following GEMM that reads bf16 operands: C16 with
  // EPI_STORE / EPI_RESID, H16 with EPI_SWIGLU_FWD
  __nv_bfloat16* C16 = nullptr;
  __nv_bfloat16* H16 = nullptr;
  // EPI_PAIR_GRU: biases of the two halves, recurrent state, residual stream
  const float* b0 = nullptr;
  const float* b1 = nullptr;
  float* state = nullptr;
  float* xres = nullptr;
  // RMSNorm of the finished rows (EPI_ACCUM / EPI_RESID / EPI_STORE, and
  // EPI_PAIR_GRU on its residual stream): ny = x * rsqrt(mean(x^2) + eps) * nw,
  // written by the kernel that sums the split-K partials (one CTA per row),
  // so the next sublayer's normalisation costs no launch of its own
  const float* nw = nullptr;
  float* ny = nullptr;
  float eps = 0.0f;
  // EPI_STORE only: leave the split-K partial planes unsummed for the
  // caller's own kernel. On return *planes_out holds the first plane
  // ([M, ldc] each, M * N floats apart, summed in index order) and
  // *splits_out their count; 1 means C itself holds the result.
  int* splits_out = nullptr;
  const float** planes_out = nullptr;
  // decode steps, with ny (EPI_ACCUM / EPI_RESID / EPI_STORE): the next
  // sublayer's causal-conv step on the normalised row (conv_step.cuh),
  // its output row into conv_out ([M, N]); ring: [M][14][N], pos: device scalar
  const float* cw3 = nullptr;
  const float* cw7 = nullptr;
  const float* cw15 = nullptr;
  float* ring = nullptr;
  const int* pos = nullptr;
  float* conv_out = nullptr;
};

// Launch. Both operands fp32 (3xTF32 or bf16-rounded per `precision`) or
// both bf16 (one kind::f16 MMA per 16-deep slice from bf16 tiles). `b_pair_off` > 0 makes every B tile two halves of BN/2 rows taken at
// logical rows n0 and n0 + b_pair_off (used to pair gate/up weights so one
// accumulator tile holds both). `k_splits` = 0 picks automatically (only
// EPI_ACCUM may split K). Returns cudaSuccess or the launch error.
// Arithmetic of the products.
enum Precision : int {
  PREC_TF32X3 = 0,  // fp32-accurate: hi*lo + lo*hi + hi*hi tf32 MMAs
  PREC_BF16 = 1,    // operands rounded to bf16, fp32 accumulation, one MMA
};

cudaError_t gemm_tf32x3(cudaStream_t stream, int M, int N, int K, const Operand& A,
                        const Operand& B, const Epilogue& epi, int b_pair_off = 0,
                        int k_splits = 0, unsigned* err_word = nullptr,
                        int precision = PREC_TF32X3);

// Number of SMs of the current device (cached).
int num_sms();

// fp32 tiled tensor map of `rank` (<= 5) dimensions, innermost first:
// dims[i] elements, stride_bytes[i] between consecutive indices of dimension
// i + 1, box[i] elements per copy; out-of-range elements read as zero.
bool encode_map_f32(CUtensorMap* m, const float* base, int rank, const uint64_t* dims,
                    const uint64_t* stride_bytes, const uint32_t* box);

// Grow the split-K workspace of `stream` on the current device to at least
// `floats` (call before capturing short-M GEMMs into a CUDA graph; calls made
// while capturing never allocate and run unsplit when the workspace is short).
cudaError_t reserve_workspace(cudaStream_t stream, size_t floats);

// Reason of the last failed gemm_tf32x3 call on this thread ("" if none).
const char* gemm_last_reason();

// 0 = automatic CTA group choice, 1 / 2 = force single CTAs / CTA pairs.
void set_force_cta_group(int cg);

}  // namespace rnet_gemm
