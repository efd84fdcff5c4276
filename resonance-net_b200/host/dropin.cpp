// C++ drop-in layer: the reference's include/layers.h, resonance_net.h and
// dist.h implemented over the C ABI (rnet_capi.h). A program written against
// the reference headers compiles against include/ here and links
// librnet_b200.so instead of the reference's objects + cuBLAS.
//
// Error behaviour follows the reference: failures print a message and exit(1)
// (layer ops, CUDA_CHECK in include/layers.h:7-14) or abort() (distributed
// init, src/dist.cpp:16-22); the C ABI underneath returns status codes.
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "dist.h"
#include "layers.h"
#include "resonance_net.h"
#include "rnet_capi.h"

namespace rnet {

namespace {

void die(int rc, const char* what) {
  if (rc != RNET_OK) {
    fprintf(stderr, "rnet error in %s (%d): %s\n", what, rc, rnet_last_error());
    exit(1);
  }
}

void* S(cudaStream_t s) { return (void*)s; }

}  // namespace

// ------------------------------------------------------------------ layers.h
void rms_norm_forward(const float* x, const float* w, float* y, float* rms_cache, int batch_seq,
                      int dim, float eps, cudaStream_t stream) {
  die(rnet_rms_norm_forward(x, w, y, rms_cache, batch_seq, dim, eps, S(stream)),
      "rms_norm_forward");
}
void rms_norm_backward(const float* dy, const float* x, const float* w, const float* rms_cache,
                       float* dx, float* dw, int batch_seq, int dim, cudaStream_t stream) {
  die(rnet_rms_norm_backward(dy, x, w, rms_cache, dx, dw, batch_seq, dim, S(stream)),
      "rms_norm_backward");
}
void embed_forward(const int* tokens, const float* table, float* output, int batch_seq,
                   int vocab, int dim, cudaStream_t stream) {
  die(rnet_embed_forward(tokens, table, output, batch_seq, vocab, dim, S(stream)),
      "embed_forward");
}
void embed_backward(const float* dout, const int* tokens, float* dtable, int batch_seq,
                    int vocab, int dim, cudaStream_t stream) {
  die(rnet_embed_backward(dout, tokens, dtable, batch_seq, vocab, dim, S(stream)),
      "embed_backward");
}
void linear_forward(const float* input, const float* weight, float* output, int M, int N, int K,
                    cublasHandle_t, cudaStream_t stream) {
  die(rnet_linear_forward(input, weight, output, M, N, K, S(stream)), "linear_forward");
}
void causal_conv_forward(const float* x, float* y, const CausalConvParams& p, float* conv_buf,
                         int batch, int seq_len, int dim, cublasHandle_t, cudaStream_t stream) {
  die(rnet_causal_conv_forward(x, y, p.conv3_w, p.conv7_w, p.conv15_w, p.mix_w, conv_buf, batch,
                               seq_len, dim, S(stream)),
      "causal_conv_forward");
}
void causal_conv_backward(const float* dy, const float* x, const CausalConvParams& p,
                          const float* conv_buf, float* dx, CausalConvParams& dp, int batch,
                          int seq_len, int dim, cublasHandle_t, cudaStream_t stream) {
  die(rnet_causal_conv_backward(dy, x, p.conv3_w, p.conv7_w, p.conv15_w, p.mix_w, conv_buf, dx,
                                dp.conv3_w, dp.conv7_w, dp.conv15_w, dp.mix_w, batch, seq_len,
                                dim, /*dmix_quirk=*/1, S(stream)),
      "causal_conv_backward");
}
void min_gru_forward(const float* x, float* y, const MinGRUParams& p, float* z_cache,
                     float* h_cache, int batch, int seq_len, int dim, cublasHandle_t,
                     cudaStream_t stream) {
  die(rnet_min_gru_forward(x, y, p.Wz, p.Wh, p.bz, p.bh, z_cache, h_cache, batch, seq_len, dim,
                           S(stream)),
      "min_gru_forward");
}
void min_gru_backward(const float* dy, const float* x, const MinGRUParams& p,
                      const float* z_cache, const float* h_cache, float* dx, MinGRUParams& dp,
                      int batch, int seq_len, int dim, cublasHandle_t, cudaStream_t stream) {
  die(rnet_min_gru_backward(dy, x, p.Wz, p.Wh, p.bz, p.bh, z_cache, h_cache, dx, dp.Wz, dp.Wh,
                            dp.bz, dp.bh, batch, seq_len, dim, S(stream)),
      "min_gru_backward");
}
void slot_memory_forward(const float* x, float* y, const SlotMemoryParams& p, float* q_cache,
                         float* scores_cache, int* topk_idx_cache, float* topk_w_cache,
                         int batch, int seq_len, int dim, int n_slots, int top_k,
                         cublasHandle_t, cudaStream_t stream) {
  die(rnet_slot_memory_forward(x, y, p.slot_keys, p.slot_values, p.proj_q, p.proj_out, q_cache,
                               scores_cache, topk_idx_cache, topk_w_cache, batch, seq_len, dim,
                               n_slots, top_k, S(stream)),
      "slot_memory_forward");
}
void slot_memory_backward(const float* dy, const float* x, const SlotMemoryParams& p,
                          const float* q_cache, const float* scores_cache,
                          const int* topk_idx_cache, const float* topk_w_cache, float* dx,
                          SlotMemoryParams& dp, int batch, int seq_len, int dim, int n_slots,
                          int top_k, cublasHandle_t, cudaStream_t stream) {
  die(rnet_slot_memory_backward(dy, x, p.slot_keys, p.slot_values, p.proj_q, p.proj_out, q_cache,
                                scores_cache, topk_idx_cache, topk_w_cache, dx, dp.slot_keys,
                                dp.slot_values, dp.proj_q, dp.proj_out, batch, seq_len, dim,
                                n_slots, top_k, S(stream)),
      "slot_memory_backward");
}
void swiglu_forward(const float* x, float* y, const SwiGLUParams& p, float* gate_cache,
                    float* up_cache, int batch_seq, int dim, int d_ff, cublasHandle_t,
                    cudaStream_t stream) {
  die(rnet_swiglu_forward(x, y, p.gate_w, p.up_w, p.down_w, gate_cache, up_cache, batch_seq, dim,
                          d_ff, S(stream)),
      "swiglu_forward");
}
void swiglu_backward(const float* dy, const float* x, const SwiGLUParams& p,
                     const float* gate_cache, const float* up_cache, float* dx, SwiGLUParams& dp,
                     int batch_seq, int dim, int d_ff, cublasHandle_t, cudaStream_t stream) {
  die(rnet_swiglu_backward(dy, x, p.gate_w, p.up_w, p.down_w, gate_cache, up_cache, dx,
                           dp.gate_w, dp.up_w, dp.down_w, batch_seq, dim, d_ff, S(stream)),
      "swiglu_backward");
}
void cross_entropy_forward(const float* logits, const int* targets, float* loss, float* dlogits,
                           int batch_seq, int vocab, cudaStream_t stream) {
  die(rnet_cross_entropy_forward(logits, targets, loss, dlogits, batch_seq, vocab, S(stream)),
      "cross_entropy_forward");
}
void residual_add(float* x, const float* y, int n, cudaStream_t stream) {
  die(rnet_residual_add(x, y, (size_t)n, S(stream)), "residual_add");
}
void scale_grads(float* grads, float scale, int n, cudaStream_t stream) {
  die(rnet_scale_grads(grads, scale, (size_t)n, S(stream)), "scale_grads");
}

// ------------------------------------------------------------------ resonance_net.h
static rnet_model_config to_c(const ModelConfig& c) {
  rnet_model_config r;
  r.d_model = c.d_model;
  r.n_layers = c.n_layers;
  r.d_ff = c.d_ff;
  r.n_heads = c.n_heads;
  r.gru_dim = c.gru_dim;
  r.n_slots = c.n_slots;
  r.slot_top_k = c.slot_top_k;
  r.vocab_size = c.vocab_size;
  r.seq_len = c.seq_len;
  r.rms_eps = c.rms_eps;
  return r;
}

static ModelConfig from_c(const rnet_model_config& r) {
  ModelConfig c;
  c.d_model = r.d_model;
  c.n_layers = r.n_layers;
  c.d_ff = r.d_ff;
  c.n_heads = r.n_heads;
  c.gru_dim = r.gru_dim;
  c.n_slots = r.n_slots;
  c.slot_top_k = r.slot_top_k;
  c.vocab_size = r.vocab_size;
  c.seq_len = r.seq_len;
  c.rms_eps = r.rms_eps;
  return c;
}

void ResonanceNet::bind_views() {
  float *p = nullptr, *g = nullptr;
  die(rnet_model_device_buffers(model_, &p, &g), "device_buffers");
  void* s = nullptr;
  die(rnet_model_stream(model_, &s), "stream");
  stream_ = (cudaStream_t)s;
  size_t n = 0;
  die(rnet_model_param_count(model_, &n), "param_count");
  total_params_ = n;
  const size_t D = cfg_.d_model, V = cfg_.vocab_size, F = cfg_.d_ff, NS = cfg_.n_slots;
  auto fill = [&](float* base, std::vector<LayerWeights>& out) {
    float* q = base + 2 * V * D + D;
    auto take = [&](size_t k) { float* r = q; q += k; return r; };
    out.resize(cfg_.n_layers);
    for (auto& w : out) {
      w.norm1_w = take(D); w.norm2_w = take(D); w.norm3_w = take(D); w.norm4_w = take(D);
      w.conv.conv3_w = take(3 * D); w.conv.conv7_w = take(7 * D);
      w.conv.conv15_w = take(15 * D); w.conv.mix_w = take(D * D);
      w.gru.Wz = take(D * D); w.gru.Wh = take(D * D); w.gru.bz = take(D); w.gru.bh = take(D);
      w.slot.slot_keys = take(D * NS); w.slot.slot_values = take(D * NS);
      w.slot.proj_q = take(D * D); w.slot.proj_out = take(D * D);
      w.ffn.gate_w = take(F * D); w.ffn.up_w = take(F * D); w.ffn.down_w = take(D * F);
    }
  };
  fill(p, layers_);
  fill(g, grads_);
}

bool ResonanceNet::init(const ModelConfig& cfg) {
  cfg_ = cfg;
  int dev = 0;
  cudaGetDevice(&dev);
  rnet_model_config c = to_c(cfg);
  int rc = rnet_model_create(&c, dev, /*reference_init=*/1, &model_);
  if (rc != RNET_OK) {
    fprintf(stderr, "ResonanceNet::init failed: %s\n", rnet_last_error());
    model_ = nullptr;
    return false;
  }
  bind_views();
  printf("ResonanceNet (sm_100a) init: d=%d, layers=%d, ff=%d, slots=%d, vocab=%d, params=%zu\n",
         cfg.d_model, cfg.n_layers, cfg.d_ff, cfg.n_slots, cfg.vocab_size, total_params_);
  return true;
}

void ResonanceNet::destroy() {
  if (model_) rnet_model_destroy(model_);
  model_ = nullptr;
  layers_.clear();
  grads_.clear();
}

void ResonanceNet::forward(const int* d_tokens, float* d_logits, int batch, int seq_len) {
  die(rnet_model_forward(model_, d_tokens, d_logits, batch, seq_len), "ResonanceNet::forward");
}

void ResonanceNet::backward(const float* d_dlogits, const int* d_tokens, int batch, int seq_len) {
  die(rnet_model_backward(model_, d_dlogits, d_tokens, batch, seq_len), "ResonanceNet::backward");
}

void ResonanceNet::step(const TrainConfig& tcfg, int) {
  die(rnet_model_step(model_, tcfg.lr, tcfg.grad_clip), "ResonanceNet::step");
}

void ResonanceNet::set_dist(DistState* dist) {
  dist_ = dist;
  if (model_)
    die(rnet_model_set_dist(model_, (dist && dist->active()) ? dist->comm : nullptr), "set_dist");
}

void ResonanceNet::zero_grad() { die(rnet_model_zero_grad(model_), "ResonanceNet::zero_grad"); }

bool ResonanceNet::save(const std::string& path) {
  if (!model_) return false;
  return rnet_model_save(model_, path.c_str()) == RNET_OK;
}

// Like the reference (src/resonance_net.cpp:784-824): an uninitialised model
// takes its configuration from the file. Unlike it, a short or mismatched
// file is rejected (returns false) instead of silently loading garbage.
bool ResonanceNet::load(const std::string& path) {
  if (!model_) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (rnet_model_create_from_checkpoint(path.c_str(), dev, &model_) != RNET_OK) {
      model_ = nullptr;
      return false;
    }
    rnet_model_config c;
    rnet_model_get_config(model_, &c);
    cfg_ = from_c(c);
    bind_views();
    if (dist_) set_dist(dist_);
    return true;
  }
  return rnet_model_load_weights(model_, path.c_str()) == RNET_OK;
}

// Declared by the reference (include/resonance_net.h:82-83) but never
// defined there. Here: prefill the prompt with the chunked scan, then one
// recurrent step per token carrying the O(1) state, all on the device (the
// steps replay one captured CUDA graph). temperature <= 0 is greedy;
// otherwise the next token follows the reference infer loop's rule
// (src/main.cpp:327-360: softmax at `temperature`, top-p 0.9 nucleus),
// sampled on the device with a fixed seed (42).
void ResonanceNet::generate(const int* prompt, int prompt_len, int* output, int max_tokens,
                            float temperature) {
  if (!model_ || prompt_len <= 0 || max_tokens <= 0) return;
  rnet_decoder* dec = nullptr;
  die(rnet_decoder_create(model_, 1, &dec), "generate: decoder");
  die(rnet_decoder_set_sampling(dec, temperature > 0.f ? temperature : 0.f, 0.9f, 42ull),
      "generate: sampling");
  int* d_tok = nullptr;
  CUDA_CHECK(cudaMalloc(&d_tok, sizeof(int) * (prompt_len > max_tokens ? prompt_len : max_tokens)));
  CUDA_CHECK(cudaMemcpy(d_tok, prompt, sizeof(int) * prompt_len, cudaMemcpyHostToDevice));
  die(rnet_decoder_prefill(dec, d_tok, prompt_len), "generate: prefill");
  // the first token comes from the prefill; each further one from a step
  int next = 0;
  die(rnet_decoder_outputs_host(dec, nullptr, &next), "generate: outputs");
  output[0] = next;
  if (max_tokens > 1) {
    die(rnet_decoder_generate(dec, max_tokens - 1, d_tok, 1), "generate: decode");
    CUDA_CHECK(cudaMemcpy(output + 1, d_tok, sizeof(int) * (max_tokens - 1),
                          cudaMemcpyDeviceToHost));
  }
  cudaFree(d_tok);
  rnet_decoder_destroy(dec);
}

// ------------------------------------------------------------------ dist.h
namespace {

int env_int(const char* name, int defval) {
  const char* s = std::getenv(name);
  if (!s || !*s) return defval;
  return std::atoi(s);
}

}  // namespace

DistState dist_init_from_env() {
  DistState st;
  st.world_size = env_int("WORLD_SIZE", 1);
  st.rank = env_int("RANK", 0);
  st.local_rank = env_int("LOCAL_RANK", st.rank);
  cudaError_t ce = cudaSetDevice(st.local_rank);
  if (st.world_size <= 1) return st;
  if (ce != cudaSuccess) {
    fprintf(stderr, "cudaSetDevice(%d) failed: %s\n", st.local_rank, cudaGetErrorString(ce));
    std::abort();
  }
  const char* uid_path = std::getenv("NCCL_UID_PATH");
  if (!uid_path) {
    fprintf(stderr, "NCCL_UID_PATH env var not set\n");
    std::abort();
  }
  unsigned char uid[128];
  int rc;
  if (st.rank == 0) {
    rc = rnet_dist_unique_id(uid);
    if (rc == RNET_OK) rc = rnet_dist_uid_file_write(uid_path, uid);
  } else {
    rc = rnet_dist_uid_file_read(uid_path, 120000, uid);
  }
  if (rc == RNET_OK) rc = rnet_dist_create(st.rank, st.world_size, st.local_rank, uid, 120000,
                                           &st.comm);
  if (rc != RNET_OK) {
    fprintf(stderr, "rank %d: distributed init failed: %s\n", st.rank, rnet_last_error());
    std::abort();
  }
  return st;
}

void dist_destroy(DistState& st) {
  if (st.comm) rnet_dist_destroy(st.comm);
  st.comm = nullptr;
  st.world_size = 1;
}

void dist_allreduce_sum(DistState& st, float* buf, size_t count, cudaStream_t stream) {
  if (!st.active()) return;
  int rc = rnet_dist_allreduce_sum(st.comm, buf, count, S(stream));
  if (rc != RNET_OK) {
    fprintf(stderr, "NCCL all-reduce failed: %s\n", rnet_last_error());
    std::abort();
  }
}

void dist_group_start(DistState& st) {
  if (st.active() && rnet_dist_group_start(st.comm) != RNET_OK) std::abort();
}
void dist_group_end(DistState& st) {
  if (st.active() && rnet_dist_group_end(st.comm) != RNET_OK) std::abort();
}

}  // namespace rnet
