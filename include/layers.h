// Drop-in replacement for the reference's include/layers.h:28-153.
//
// Same namespace, function names, argument order and meaning, and the same
// accumulate / overwrite contract; the implementations run on librnet_b200.so
// (sm_100a kernels through the C ABI in rnet_capi.h). The cublasHandle_t
// parameters are kept for source compatibility and ignored. On a failing call
// the functions print the library's message and exit(1), as the reference's
// CUDA_CHECK does.
#pragma once
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "config.h"

#define CUDA_CHECK(call)                                                                  \
  do {                                                                                    \
    cudaError_t err = (call);                                                             \
    if (err != cudaSuccess) {                                                             \
      fprintf(stderr, "CUDA error at %s:%d: %s\n", __FILE__, __LINE__,                    \
              cudaGetErrorString(err));                                                   \
      exit(1);                                                                            \
    }                                                                                     \
  } while (0)

#define CUBLAS_CHECK(call)                                                                \
  do {                                                                                    \
    cublasStatus_t st = (call);                                                           \
    if (st != CUBLAS_STATUS_SUCCESS) {                                                    \
      fprintf(stderr, "cuBLAS error at %s:%d: %d\n", __FILE__, __LINE__, (int)st);         \
      exit(1);                                                                            \
    }                                                                                     \
  } while (0)

namespace rnet {

// ---- RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w ----------------------------
void rms_norm_forward(const float* x, const float* w, float* y, float* rms_cache, int batch_seq,
                      int dim, float eps, cudaStream_t stream);
// dx overwritten, dw accumulated.
void rms_norm_backward(const float* dy, const float* x, const float* w, const float* rms_cache,
                       float* dx, float* dw, int batch_seq, int dim, cudaStream_t stream);

// ---- Embedding / output projection -----------------------------------------
void embed_forward(const int* tokens, const float* table, float* output, int batch_seq,
                   int vocab, int dim, cudaStream_t stream);
void embed_backward(const float* dout, const int* tokens, float* dtable, int batch_seq,
                    int vocab, int dim, cudaStream_t stream);
// output[M,N] = input[M,K] * weight[N,K]^T
void linear_forward(const float* input, const float* weight, float* output, int M, int N, int K,
                    cublasHandle_t cublas, cudaStream_t stream);

// ---- Multi-scale causal convolution (k = 3, 7, 15) + mix --------------------
struct CausalConvParams {
  float* conv3_w;   // [3, d_model]
  float* conv7_w;   // [7, d_model]
  float* conv15_w;  // [15, d_model]
  float* mix_w;     // [d_model, d_model]
};
// conv_buf [3, B*T, D] receives {c3 + c7 + c15, c7, c15}.
void causal_conv_forward(const float* x, float* y, const CausalConvParams& p, float* conv_buf,
                         int batch, int seq_len, int dim, cublasHandle_t cublas,
                         cudaStream_t stream);
// dx and all parameter gradients accumulated. The mix-weight gradient uses the
// reference's operand (c3 + c7 + c15 re-summed over the cached buffer).
void causal_conv_backward(const float* dy, const float* x, const CausalConvParams& p,
                          const float* conv_buf, float* dx, CausalConvParams& dp, int batch,
                          int seq_len, int dim, cublasHandle_t cublas, cudaStream_t stream);

// ---- MinGRU: h_t = (1 - z) h_{t-1} + z h~, z = sigmoid(x Wz^T + bz) ---------
struct MinGRUParams {
  float* Wz;  // [d_model, d_model]
  float* Wh;  // [d_model, d_model]
  float* bz;  // [d_model]
  float* bh;  // [d_model]
};
void min_gru_forward(const float* x, float* y, const MinGRUParams& p, float* z_cache,
                     float* h_cache, int batch, int seq_len, int dim, cublasHandle_t cublas,
                     cudaStream_t stream);
void min_gru_backward(const float* dy, const float* x, const MinGRUParams& p,
                      const float* z_cache, const float* h_cache, float* dx, MinGRUParams& dp,
                      int batch, int seq_len, int dim, cublasHandle_t cublas,
                      cudaStream_t stream);

// ---- Slot memory: top-k sparse read of learned slots -------------------------
struct SlotMemoryParams {
  float* slot_keys;    // [d_model, n_slots]
  float* slot_values;  // [d_model, n_slots]
  float* proj_q;       // [d_model, d_model]
  float* proj_out;     // [d_model, d_model]
};
void slot_memory_forward(const float* x, float* y, const SlotMemoryParams& p, float* q_cache,
                         float* scores_cache, int* topk_idx_cache, float* topk_w_cache,
                         int batch, int seq_len, int dim, int n_slots, int top_k,
                         cublasHandle_t cublas, cudaStream_t stream);
void slot_memory_backward(const float* dy, const float* x, const SlotMemoryParams& p,
                          const float* q_cache, const float* scores_cache,
                          const int* topk_idx_cache, const float* topk_w_cache, float* dx,
                          SlotMemoryParams& dp, int batch, int seq_len, int dim, int n_slots,
                          int top_k, cublasHandle_t cublas, cudaStream_t stream);

// ---- SwiGLU FFN (row-major gate, up [d_ff, d_model]; down [d_model, d_ff]) ---
struct SwiGLUParams {
  float* gate_w;
  float* up_w;
  float* down_w;
};
void swiglu_forward(const float* x, float* y, const SwiGLUParams& p, float* gate_cache,
                    float* up_cache, int batch_seq, int dim, int d_ff, cublasHandle_t cublas,
                    cudaStream_t stream);
void swiglu_backward(const float* dy, const float* x, const SwiGLUParams& p,
                     const float* gate_cache, const float* up_cache, float* dx, SwiGLUParams& dp,
                     int batch_seq, int dim, int d_ff, cublasHandle_t cublas,
                     cudaStream_t stream);

// ---- Loss / utilities --------------------------------------------------------
// *loss = sum over tokens (overwritten); dlogits = softmax - onehot.
void cross_entropy_forward(const float* logits, const int* targets, float* loss, float* dlogits,
                           int batch_seq, int vocab, cudaStream_t stream);
void residual_add(float* x, const float* y, int n, cudaStream_t stream);
void scale_grads(float* grads, float scale, int n, cudaStream_t stream);

}  // namespace rnet
