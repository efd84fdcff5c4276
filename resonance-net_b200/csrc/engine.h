// ResonanceNet model engine: parameters, gradients, activation caches and the
// per-layer forward / backward / SGD schedule on one CUDA stream.
//
// Parameters and gradients each live in ONE flat device buffer laid out in
// checkpoint tensor order (reference src/resonance_net.cpp:759-778), so a
// checkpoint is one read/write, the optimizer is one pass, and data-parallel
// gradient buckets are contiguous ranges. Within a layer Wz|Wh and gate|up
// are adjacent in that order, which the fused GEMMs use as [2D,D] / [2F,D].
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <string>
#include <vector>

#include "../../include/rnet_capi.h"

namespace rnet_engine {

struct LayerParams {
  float *n1, *n2, *n3, *n4, *c3, *c7, *c15, *mix, *Wz, *Wh, *bz, *bh, *keys, *vals, *pq, *pout,
      *gate, *up, *down;
  size_t offset, count;  // range of this layer in the flat buffer
};

struct LayerAct {
  float *n1, *n2, *n3, *n4;
  float *rinv1, *rinv2, *rinv3, *rinv4;
  float *S, *Sq;
  float *P;  // [N, 2D] = pz | ph
  float *z, *h;
  float *q, *r;
  int* idx;
  float* w;
  float *r1, *r2, *r3;
  float *G, *U, *H;
};

class DistComm;  // dist.cu

class Engine {
 public:
  explicit Engine(const rnet_model_config& c);
  ~Engine();
  int init(int device, bool reference_init);  // allocate + initialise weights

  // Parameters
  size_t param_count() const { return P_; }
  float* params() { return params_; }
  float* grads() { return grads_; }
  int set_params_host(const float* h, size_t n);
  int get_params_host(float* h, size_t n);
  int get_grads_host(float* h, size_t n);
  int refresh_shadows();  // transposed key/value copies after a weight change

  int forward(const int* d_tokens, float* d_logits, int B, int T);
  int backward(const float* d_dlogits, const int* d_tokens, int B, int T);
  int zero_grad();
  int step(float lr, float clip);
  // zero_grad + forward + CE (dlogits scaled by 1/N) + backward + step.
  // d_loss_sum: device float receiving sum of token losses (may be null).
  int train_step(const int* d_in, const int* d_tgt, int B, int T, float lr, float clip,
                 float* d_loss_sum);

  int save(const char* path);
  int load_weights(const char* path);  // config in file must match

  int topk(int layer, int** idx, float** w);
  cudaStream_t stream() const { return stream_; }
  const rnet_model_config& config() const { return cfg_; }

  bool conv_quirk = true;  // reference dmix operand (S + c7 + c15)
  DistComm* dist = nullptr;

  // workspace capacity in tokens
  int ensure_capacity(int N, bool with_caches);

 private:
  int gemm_err(cudaError_t e, const char* what);
  int layer_forward(int l, const float* Xl, float* Xn, LayerAct& a, int B, int T);
  int layer_backward(int l, int B, int T);
  int head_backward(const float* d_dlogits, int N);

  rnet_model_config cfg_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  size_t P_ = 0;
  float* params_ = nullptr;
  float* grads_ = nullptr;
  float *embed_, *outw_, *fnorm_, *g_embed_, *g_outw_, *g_fnorm_;
  std::vector<LayerParams> W_, G_;
  float* KT_ = nullptr;  // [L][S][D]
  float* VT_ = nullptr;
  float* dKT_ = nullptr;
  float* dVT_ = nullptr;
  float* scratch_ = nullptr;  // sgd / ce scratch
  float* loss_dev_ = nullptr;
  float* norm_dev_ = nullptr;

  // activation arena
  void* arena_ = nullptr;
  size_t arena_bytes_ = 0;
  int cap_N_ = 0;
  bool cap_caches_ = false;
  std::vector<LayerAct> act_;
  float* X_ = nullptr;  // [L+1][N][D]
  float *nf_, *rinvf_, *dlogits_, *logits_;
  float *dX_, *dsub_, *dS_, *dq_, *dr_, *dPZH_, *dGU_, *dnf_, *conv_parts_, *scores_;
  bool have_cache_ = false;
  int last_B_ = 0, last_T_ = 0;
};

}  // namespace rnet_engine
