// Drop-in replacement for the reference's include/config.h (ModelConfig,
// TrainConfig). ModelConfig's first 40 bytes are the checkpoint header, so its
// data members keep the reference's order and types exactly.
#pragma once
#include <cstddef>
#include <string>

namespace rnet {

struct ModelConfig {
  int d_model = 512;
  int n_layers = 8;
  int d_ff = 1024;
  int n_heads = 8;    // unused by the layer math (kept for the header layout)
  int gru_dim = 512;  // unused by the layer math (kept for the header layout)
  int n_slots = 1024;
  int slot_top_k = 2;
  int vocab_size = 256;
  int seq_len = 256;
  float rms_eps = 1e-6f;

  // Depthwise causal convolution scales.
  static constexpr int CONV_SCALES = 3;
  static constexpr int conv_kernels[CONV_SCALES] = {3, 7, 15};

  int head_dim() const { return d_model / n_heads; }

  // Number of fp32 parameters (= floats after the 40-byte checkpoint header).
  size_t param_count() const {
    const size_t D = d_model, F = d_ff, S = n_slots, V = vocab_size;
    const size_t per_layer = 4 * D                  // RMSNorm gains
                             + (3 + 7 + 15) * D     // depthwise taps
                             + D * D                // conv mix
                             + 2 * D * D + 2 * D    // MinGRU Wz, Wh, bz, bh
                             + 2 * D * S + 2 * D * D  // slot keys, values, proj_q, proj_out
                             + 3 * D * F;           // SwiGLU gate, up, down
    return 2 * V * D + D + per_layer * (size_t)n_layers;
  }
};

struct TrainConfig {
  float lr = 3e-4f;
  float grad_clip = 1.0f;
  int batch_size = 64;
  int max_steps = 100000;
  int warmup_steps = 1000;  // parsed by the reference CLI but never applied
  int log_interval = 10;
  int save_interval = 1000;
  int eval_interval = 100;
  int eval_tokens = 4096;
  std::string data_path;
  std::string save_path = "checkpoints/";
};

}  // namespace rnet
