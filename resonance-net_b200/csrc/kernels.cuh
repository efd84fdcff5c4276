// Launchers of the non-GEMM ResonanceNet kernels (all sm_100a, fp32).
// Every launcher is asynchronous on `s` and returns the launch status.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace rnet_k {

// Launch bookkeeping: count `n` kernels launched by this library and return
// the launch status (defined in status.cu).
cudaError_t launched(unsigned n = 1);

// ---- RMSNorm (rms_norm.cu) ------------------------------------------------
// y = x * rinv * w, rinv = rsqrt(mean(x^2) + eps)        (y may be null)
// xcopy (optional): also store x there (seeds a residual sum that a GEMM then
// accumulates into). y16 (optional): y rounded to bf16 as well (the operand
// of a following bf16 GEMM).
cudaError_t rms_norm_fwd(const float* x, const float* w, float* y, float* rinv, int rows,
                         int D, float eps, cudaStream_t s, float* xcopy = nullptr,
                         __nv_bfloat16* y16 = nullptr);
// dx_norm = rinv*(dy*w - xhat*mean(dy*w*xhat)); dw += sum_rows dy*xhat.
// mode 0: dx = dx_norm (overwrite); mode 1: dx += dx_norm (residual stream).
// dx16 (optional): the final dx rounded to bf16 as well.
cudaError_t rms_norm_bwd(const float* dy, const float* x, const float* w, const float* rinv,
                         float* dx, float* dw, int rows, int D, int mode, cudaStream_t s,
                         __nv_bfloat16* dx16 = nullptr);
// y = bf16(x), n elements (x, y 16-byte aligned when n % 8 == 0 is used).
cudaError_t to_bf16(const float* x, __nv_bfloat16* y, size_t n, cudaStream_t s);
// y = float(x), n elements.
cudaError_t from_bf16(const __nv_bfloat16* x, float* y, size_t n, cudaStream_t s);

// ---- depthwise causal convolution (causal_conv.cu) -------------------------
// c3/c7/c15 of x over each length-T sequence, S = c3 + c7 + c15.
// Writes S; optionally Sq = S + c7 + c15 (reference dmix operand) or c7, c15
// individually (reference conv_buf layout), not both. D % 4 == 0.
cudaError_t conv_fwd(const float* x, const float* w3, const float* w7, const float* w15,
                     float* S, float* Sq, float* c7, float* c15, int B, int T, int D,
                     cudaStream_t s);
// Model path with bf16 outputs: S16 (and Sq16 if given) only.
cudaError_t conv_fwd_bf16(const float* x, const float* w3, const float* w7, const float* w15,
                          __nv_bfloat16* S16, __nv_bfloat16* Sq16, int B, int T, int D,
                          cudaStream_t s);
// dx (+)= sum_K conv_K^T(dS); dw_K[k] += sum x[t-(K-1)+k] dS[t].
// accumulate: 0 -> dx = ..., 1 -> dx += ...
// `partials` is scratch of conv_bwd_partials_floats(B, T, D) floats.
size_t conv_bwd_partials_floats(int B, int T, int D);
cudaError_t conv_bwd(const float* dS, const float* x, const float* w3, const float* w7,
                     const float* w15, float* dx, float* dw3, float* dw7, float* dw15,
                     float* partials, int B, int T, int D, int accumulate, cudaStream_t s);

// ---- MinGRU scan (min_gru_scan.cu) ----------------------------------------
// z = sigmoid(pz + bz), h~ = ph + bh, h_t = (1-z) h_{t-1} + z h~ (h_{-1} = 0).
// pz/ph rows have stride ldp. Writes z, h; optional y = h (copy) and optional
// residual out = res + h. h_as_diff: the `h` output receives e_t = h~_t -
// h_{t-1} instead (all the backward needs of h~ and h; exact in fp32).
// out2 (optional): a second copy of out.
cudaError_t gru_scan_fwd(const float* pz, const float* ph, int ldp, const float* bz,
                         const float* bh, float* z, float* h, float* y, const float* res,
                         float* out, int B, int T, int D, cudaStream_t s, bool h_as_diff = false,
                         float* out2 = nullptr);
// Reverse scan: dh_t = dy_t + (1 - z_{t+1}) dh_{t+1};
// dz = dh (h~ - h_{t-1}) z (1-z), dh~ = dh z. h~ = ph + bh (ph stride ldp).
// ph == nullptr: `h` holds e = h~ - h_{t-1} from gru_scan_fwd(h_as_diff) and
// bh is not read.
// Writes dz/dh~ with row stride ldd (dh~ at column offset `dht_off`),
// dbz += sum dz, dbh += sum dh~.
// dzh16 (optional): dz / dh~ as bf16 into dzh16 (same row stride ldd, dh~ at
// the same column offset as dht - dz); dz, dht are then not written.
cudaError_t gru_scan_bwd(const float* dy, const float* z, const float* h, const float* ph,
                         int ldp, const float* bh, float* dz, float* dht, int ldd, float* dbz,
                         float* dbh, int B, int T, int D, cudaStream_t s,
                         __nv_bfloat16* dzh16 = nullptr);

// ---- slot memory (slot_memory.cu) -----------------------------------------
// out[j*R + i] = in[i*C + j] (+ accumulate into out if acc)
cudaError_t transpose(const float* in, float* out, int R, int C, int acc, cudaStream_t s);
// A batch of 2 * pairs transposes in one launch: matrix (p, q), q in {0, 1},
// reads in + p * in_stride2 + q * in_stride1 ([R, C]) and writes
// (q ? out1 : out0) + p * out_stride ([C, R]).
cudaError_t transpose_pairs(const float* in, size_t in_stride1, size_t in_stride2, float* out0,
                            float* out1, size_t out_stride, int pairs, int R, int C, int acc,
                            cudaStream_t s);
// r[n,:] = sum_j w[n,j] VT[idx[n,j], :]   (r16: bf16 copy; r may be null then)
cudaError_t slot_gather(const int* idx, const float* w, const float* VT, float* r, int N,
                        int D, int S, int k, unsigned* err, cudaStream_t s,
                        __nv_bfloat16* r16 = nullptr);
// Sparse backward through top-k + softmax + gather (one warp per token):
//   dwj = <dr, VT[idx_j]>, dsc_j = w_j (dwj - sum w dw), dq = sum dsc_j KT[idx_j]
//   dVT[idx_j] += w_j dr, dKT[idx_j] += dsc_j q   (dq16: bf16 dq; dq may be null then)
cudaError_t slot_sparse_bwd(const float* dr, const int* idx, const float* w, const float* VT,
                            const float* KT, const float* q, float* dq, float* dVT, float* dKT,
                            int N, int D, int S, int k, unsigned* err, cudaStream_t s,
                            __nv_bfloat16* dq16 = nullptr);
// Top-k (k <= 8) over a materialised score matrix, reference order semantics,
// + softmax (used by the per-op API for k != 2).
cudaError_t topk_rows(const float* scores, int* idx, float* w, int N, int S, int k,
                      cudaStream_t s);

// ---- embedding / loss / utilities (embed_loss.cu) -------------------------
cudaError_t embed_fwd(const int* tok, const float* table, float* out, int N, int V, int D,
                      unsigned* err, cudaStream_t s);
cudaError_t embed_bwd(const float* dout, const int* tok, float* dtable, int N, int V, int D,
                      cudaStream_t s);
// loss_sum (overwritten) = sum_n -(log softmax(l_n)[t_n]); dl = (softmax - onehot)*scale.
// `partials` scratch: ce_partials_floats(N) floats.
size_t ce_partials_floats(int N);
cudaError_t cross_entropy(const float* logits, const int* tgt, float* loss_sum, float* dl,
                          float scale, float* partials, int N, int V, unsigned* err,
                          cudaStream_t s);
cudaError_t residual_add(float* x, const float* y, size_t n, cudaStream_t s);
cudaError_t scale(float* x, float a, size_t n, cudaStream_t s);
cudaError_t add3(const float* a, const float* b, const float* c, float* out, size_t n,
                 cudaStream_t s);
// h = g * sigmoid(g) * u   (reference silu_mul_kernel, src/swiglu_ffn.cu:11-21)
cudaError_t silu_mul(const float* g, const float* u, float* h, size_t n, cudaStream_t s);
// In place over dgu = [dG | dU] ([N, 2F], row stride ld) holding dH in its
// dG half: dG = dH * u * silu'(g), dU = dH * silu(g) (G, U: [N, F] caches).
// dgu16 (optional): [dG | dU] written as bf16 there (row stride ld) instead
// of in place.
cudaError_t swiglu_bwd_pointwise(float* dgu, int ld, const float* G, const float* U, int N, int F,
                                 cudaStream_t s, __nv_bfloat16* dgu16 = nullptr);

// ---- recurrent decode (decode.cu) -----------------------------------------
// The decode step's slot sublayer after the score GEMM, in one launch:
// top-2 over the scores (the sum of n_planes split-K partial planes [M, S],
// M * S floats apart, in plane order; 1 = plain scores), then
// x[row] += w0 VP[i0] + w1 VP[i1] with VP = V * proj_out^T ([S, D], see
// fold_rows) and ny[row] = RMSNorm(x[row]) * nw. S % 4 == 0, D % 4 == 0.
cudaError_t topk2_gather_residual_norm(const float* planes, int n_planes, int* idx, float* w,
                                       int M, int S, const float* VP, float* x, int D,
                                       const float* nw, float* ny, float eps, cudaStream_t s);
// out[R, J] = A[R, K] * B, B(d, j) = B[d * bd + j * bj], accumulated in double:
// folds two fixed projections into one matrix (decode: keys with proj_q,
// values with proj_out).
cudaError_t fold_rows(const float* A, const float* B, size_t bd, size_t bj, float* out, int R,
                      int J, int K, cudaStream_t s);
// ring: [M][14][D] last conv inputs indexed by position mod 14; *pos = index
// of the current token (device scalar, advanced by argmax_rows).
cudaError_t decode_conv(const float* n, float* ring, const int* pos, const float* w3,
                        const float* w7, const float* w15, float* S, int M, int D,
                        cudaStream_t s);
cudaError_t decode_extract_state(const float* n1, const float* h, float* ring, float* hs, int M,
                                 int T, int D, cudaStream_t s);
cudaError_t last_rows(const float* x, float* out, int M, int T, int D, cudaStream_t s);
cudaError_t argmax_rows(const float* logits, int M, int V, int* tok, int* out, int* pos,
                        cudaStream_t s);
// Next token per row: greedy (temperature <= 0, as argmax_rows) or
// temperature + top-p sampling with the reference infer loop's rule
// (src/main.cpp:327-360); the uniform comes from (seed, row, position of the
// sampled token = *pos + advance); advance = 1 advances *pos afterwards.
cudaError_t sample_rows(const float* logits, int M, int V, float temperature, float top_p,
                        unsigned long long seed, int* tok, int* pos, int advance, cudaStream_t s);

// ---- optimizer (optimizer.cu) ---------------------------------------------
// Global-norm clip + SGD over one flat buffer, no host synchronisation:
//   lr_eff = lr/world * min(1, clip / (||g|| / world))   (if clip > 0)
//   p -= lr_eff * g
// `scratch` = sgd_scratch_floats() floats. norm_out (optional) gets ||g||.
// params16 (optional): the updated parameters rounded to bf16 as well.
// Extensions (defaults = the reference's plain SGD): weight_decay adds
// wd * p to the gradient after clipping; velocity (n floats) turns on
// momentum: v = momentum * v + g (+ wd * p), p -= lr_eff * v.
size_t sgd_scratch_floats();
cudaError_t sgd_clip_step(float* params, const float* grads, size_t n, float lr, float clip,
                          int world, float* scratch, float* norm_out, cudaStream_t s,
                          __nv_bfloat16* params16 = nullptr, float* velocity = nullptr,
                          float momentum = 0.0f, float weight_decay = 0.0f);

}  // namespace rnet_k
