// Drop-in replacement for the reference's include/resonance_net.h:11-131.
//
// Same public interface (init / forward / backward / step / zero_grad /
// save / load / set_dist / generate / config / param_count) and the same
// checkpoint byte layout. The weights, gradients and caches live in
// librnet_b200.so; LayerWeights / LayerGrads expose device pointers into its
// flat parameter / gradient buffers in the reference's field names.
#pragma once
#include <string>
#include <vector>

#include "config.h"
#include "layers.h"

struct rnet_model;

namespace rnet {

struct DistState;

struct LayerWeights {
  float* norm1_w;  // pre-conv
  float* norm2_w;  // pre-gru
  float* norm3_w;  // pre-slot
  float* norm4_w;  // pre-ffn
  CausalConvParams conv;
  MinGRUParams gru;
  SlotMemoryParams slot;
  SwiGLUParams ffn;
};

using LayerGrads = LayerWeights;

class ResonanceNet {
 public:
  bool init(const ModelConfig& cfg);
  void destroy();

  // tokens [batch, seq] (device) -> logits [batch, seq, vocab] (device)
  void forward(const int* d_tokens, float* d_logits, int batch, int seq_len);
  // from dlogits (device), using the caches of the last forward
  void backward(const float* d_dlogits, const int* d_tokens, int batch, int seq_len);
  // clipped SGD (all-reduces gradients when a DistState is attached)
  void step(const TrainConfig& tcfg, int step_num);
  void set_dist(DistState* dist);
  void zero_grad();

  bool save(const std::string& path);
  bool load(const std::string& path);

  // Autoregressive generation with the O(1) recurrent state: prompt (host,
  // prompt_len bytes) -> output (host, max_tokens bytes). temperature <= 0
  // selects greedy argmax.
  void generate(const int* prompt, int prompt_len, int* output, int max_tokens,
                float temperature = 0.8f);

  const ModelConfig& config() const { return cfg_; }
  size_t param_count() const { return total_params_; }

  // Device views in the reference's field layout (valid after init/load).
  const std::vector<LayerWeights>& layers() const { return layers_; }
  const std::vector<LayerGrads>& grads() const { return grads_; }
  cudaStream_t stream() const { return stream_; }
  rnet_model* handle() const { return model_; }

 private:
  void bind_views();

  ModelConfig cfg_;
  rnet_model* model_ = nullptr;
  cudaStream_t stream_ = nullptr;
  size_t total_params_ = 0;
  std::vector<LayerWeights> layers_;
  std::vector<LayerGrads> grads_;
  DistState* dist_ = nullptr;
};

}  // namespace rnet
