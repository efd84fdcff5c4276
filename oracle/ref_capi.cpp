// ORACLE HARNESS — test infrastructure only (never part of librnet_b200.so).
//
// A C-ABI wrapper around the UNMODIFIED reference implementation
// (KristianPilatovich/resonance-net: src/*.cu, src/resonance_net.cpp,
// src/dist.cpp), compiled from the reference's own source files by
// oracle/Makefile into oracle/_ref/libref.so. It lets Python drive the
// reference's CUDA path on the GPU box with host buffers, to pin the CPU
// oracle and to time the reference (bench.py --impl reference).
//
// Private members of ResonanceNet are read through `#define private public`
// so gradients, top-k caches and parameters can be dumped in checkpoint order.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#define private public
#include "resonance_net.h"
#undef private
#include "dist.h"
#include "layers.h"
#include "data_loader.cpp"  // the reference's DataLoader (src/data_loader.cpp), unmodified

using namespace rnet;

namespace {

struct Handle {
  ResonanceNet model;
  int* d_in = nullptr;
  int* d_tgt = nullptr;
  float* d_logits = nullptr;
  float* d_dlogits = nullptr;
  float* d_loss = nullptr;
  int cap = 0;
  void ensure(int BS) {
    if (BS <= cap) return;
    if (d_in) { cudaFree(d_in); cudaFree(d_tgt); cudaFree(d_logits); cudaFree(d_dlogits); }
    const int V = model.cfg_.vocab_size;
    cudaMalloc(&d_in, sizeof(int) * BS);
    cudaMalloc(&d_tgt, sizeof(int) * BS);
    cudaMalloc(&d_logits, sizeof(float) * (size_t)BS * V);
    cudaMalloc(&d_dlogits, sizeof(float) * (size_t)BS * V);
    if (!d_loss) cudaMalloc(&d_loss, sizeof(float));
    cap = BS;
  }
};

// Visit (pointer, count) of every parameter (or gradient) tensor in
// checkpoint order (src/resonance_net.cpp:759-778).
template <class F>
void visit(ResonanceNet& m, bool grads, F f) {
  const ModelConfig& c = m.cfg_;
  const size_t D = c.d_model, V = c.vocab_size, FF = c.d_ff, NS = c.n_slots;
  f(grads ? m.d_embed_g_ : m.d_embed_w_, V * D);
  f(grads ? m.d_output_g_ : m.d_output_w_, V * D);
  f(grads ? m.d_final_norm_g_ : m.d_final_norm_, D);
  for (int l = 0; l < c.n_layers; ++l) {
    if (!grads) {
      auto& w = m.layers_[l];
      f(w.norm1_w, D); f(w.norm2_w, D); f(w.norm3_w, D); f(w.norm4_w, D);
      f(w.conv.conv3_w, 3 * D); f(w.conv.conv7_w, 7 * D); f(w.conv.conv15_w, 15 * D);
      f(w.conv.mix_w, D * D); f(w.gru.Wz, D * D); f(w.gru.Wh, D * D); f(w.gru.bz, D);
      f(w.gru.bh, D); f(w.slot.slot_keys, D * NS); f(w.slot.slot_values, D * NS);
      f(w.slot.proj_q, D * D); f(w.slot.proj_out, D * D); f(w.ffn.gate_w, D * FF);
      f(w.ffn.up_w, D * FF); f(w.ffn.down_w, FF * D);
    } else {
      auto& w = m.grads_[l];
      f(w.norm1_w, D); f(w.norm2_w, D); f(w.norm3_w, D); f(w.norm4_w, D);
      f(w.conv.conv3_w, 3 * D); f(w.conv.conv7_w, 7 * D); f(w.conv.conv15_w, 15 * D);
      f(w.conv.mix_w, D * D); f(w.gru.Wz, D * D); f(w.gru.Wh, D * D); f(w.gru.bz, D);
      f(w.gru.bh, D); f(w.slot.slot_keys, D * NS); f(w.slot.slot_values, D * NS);
      f(w.slot.proj_q, D * D); f(w.slot.proj_out, D * D); f(w.ffn.gate_w, D * FF);
      f(w.ffn.up_w, D * FF); f(w.ffn.down_w, FF * D);
    }
  }
}

void copy_flat(ResonanceNet& m, bool grads, float* host) {
  size_t off = 0;
  visit(m, grads, [&](float* d, size_t n) {
    cudaMemcpy(host + off, d, n * sizeof(float), cudaMemcpyDeviceToHost);
    off += n;
  });
}

}  // namespace

extern "C" {

// Load a checkpoint (reference format) into a fresh reference model.
void* ref_model_load(const char* path) {
  Handle* h = new Handle();
  if (!h->model.load(path)) { delete h; return nullptr; }
  return h;
}

void ref_model_destroy(void* hp) {
  Handle* h = (Handle*)hp;
  if (!h) return;
  if (h->d_in) { cudaFree(h->d_in); cudaFree(h->d_tgt); cudaFree(h->d_logits); cudaFree(h->d_dlogits); }
  if (h->d_loss) cudaFree(h->d_loss);
  h->model.destroy();
  delete h;
}

size_t ref_model_param_count(void* hp) { return ((Handle*)hp)->model.cfg_.param_count(); }

void ref_model_get_params(void* hp, float* host) { copy_flat(((Handle*)hp)->model, false, host); }
void ref_model_get_grads(void* hp, float* host) { copy_flat(((Handle*)hp)->model, true, host); }

// One step exactly as src/main.cpp:128-152 with host token buffers.
// Returns the summed loss (main.cpp divides by BS for printing).
float ref_train_step(void* hp, const int* h_in, const int* h_tgt, int B, int T, float lr,
                     float clip) {
  Handle* h = (Handle*)hp;
  const int BS = B * T;
  h->ensure(BS);
  cudaMemcpy(h->d_in, h_in, BS * sizeof(int), cudaMemcpyHostToDevice);
  cudaMemcpy(h->d_tgt, h_tgt, BS * sizeof(int), cudaMemcpyHostToDevice);
  TrainConfig tc;
  tc.lr = lr;
  tc.grad_clip = clip;
  tc.batch_size = B;
  h->model.zero_grad();
  h->model.forward(h->d_in, h->d_logits, B, T);
  cross_entropy_forward(h->d_logits, h->d_tgt, h->d_loss, h->d_dlogits, BS,
                        h->model.cfg_.vocab_size, 0);
  scale_grads(h->d_dlogits, 1.0f / BS, BS * h->model.cfg_.vocab_size, 0);
  h->model.backward(h->d_dlogits, h->d_in, B, T);
  h->model.step(tc, 1);
  float loss = 0.0f;
  cudaMemcpy(&loss, h->d_loss, sizeof(float), cudaMemcpyDeviceToHost);
  return loss;
}

// Same step with device-resident token buffers (timing path, no host copies).
void ref_train_step_device(void* hp, const int* d_in, const int* d_tgt, int B, int T, float lr,
                           float clip) {
  Handle* h = (Handle*)hp;
  const int BS = B * T;
  h->ensure(BS);
  TrainConfig tc;
  tc.lr = lr;
  tc.grad_clip = clip;
  tc.batch_size = B;
  h->model.zero_grad();
  h->model.forward(d_in, h->d_logits, B, T);
  cross_entropy_forward(h->d_logits, d_tgt, h->d_loss, h->d_dlogits, BS,
                        h->model.cfg_.vocab_size, 0);
  scale_grads(h->d_dlogits, 1.0f / BS, BS * h->model.cfg_.vocab_size, 0);
  h->model.backward(h->d_dlogits, d_in, B, T);
  h->model.step(tc, 1);
}

// Last forward's logits [B*T, V] and per-layer top-k caches [L, B*T, k].
void ref_get_logits(void* hp, float* host, int BS) {
  Handle* h = (Handle*)hp;
  cudaMemcpy(host, h->d_logits, sizeof(float) * (size_t)BS * h->model.cfg_.vocab_size,
             cudaMemcpyDeviceToHost);
}
void ref_get_topk(void* hp, int* idx, float* w, int BS) {
  Handle* h = (Handle*)hp;
  const int k = h->model.cfg_.slot_top_k;
  for (int l = 0; l < h->model.cfg_.n_layers; ++l) {
    cudaMemcpy(idx + (size_t)l * BS * k, h->model.cache_[l].topk_idx, sizeof(int) * BS * k,
               cudaMemcpyDeviceToHost);
    cudaMemcpy(w + (size_t)l * BS * k, h->model.cache_[l].topk_w, sizeof(float) * BS * k,
               cudaMemcpyDeviceToHost);
  }
}

// Forward only (src/main.cpp:234-244 bench path) with host tokens.
void ref_forward(void* hp, const int* h_in, int B, int T, float* h_logits) {
  Handle* h = (Handle*)hp;
  const int BS = B * T;
  h->ensure(BS);
  cudaMemcpy(h->d_in, h_in, BS * sizeof(int), cudaMemcpyHostToDevice);
  h->model.forward(h->d_in, h->d_logits, B, T);
  if (h_logits) ref_get_logits(hp, h_logits, BS);
  cudaDeviceSynchronize();
}

void ref_forward_device(void* hp, const int* d_in, int B, int T) {
  Handle* h = (Handle*)hp;
  h->ensure(B * T);
  h->model.forward(d_in, h->d_logits, B, T);
}

int ref_sync(void) { return (int)cudaDeviceSynchronize(); }

}  // extern "C"

extern "C" {

// A fresh reference model initialised by its own init_weights()
// (src/resonance_net.cpp:180-216) for the given 40-byte ModelConfig.
void* ref_model_init(const ModelConfig* cfg) {
  Handle* h = new Handle();
  if (!h->model.init(*cfg)) { delete h; return nullptr; }
  return h;
}

// ResonanceNet::save (src/resonance_net.cpp:743-782). Returns 1 on success.
int ref_model_save(void* hp, const char* path) { return ((Handle*)hp)->model.save(path) ? 1 : 0; }

// ResonanceNet::load into an existing model (src/resonance_net.cpp:784-824).
int ref_model_load_into(void* hp, const char* path) {
  return ((Handle*)hp)->model.load(path) ? 1 : 0;
}

// Last forward's slot scores of one layer, [BS, n_slots] (scores_cache,
// written by src/slot_memory.cu:79-119).
void ref_get_scores(void* hp, int layer, float* host, int BS) {
  Handle* h = (Handle*)hp;
  cudaMemcpy(host, h->model.cache_[layer].scores_cache,
             sizeof(float) * (size_t)BS * h->model.cfg_.n_slots, cudaMemcpyDeviceToHost);
}

}  // extern "C"

extern "C" {

// `steps` batches from the reference's DataLoader (src/data_loader.cpp:31-52)
// seeded like src/main.cpp:117; path = corpus file, or "" for its synthetic
// tokens. inputs / targets: [steps][B*T]. Returns 1 on success.
int ref_loader_batches(const char* path, unsigned seed, int B, int T, int steps, int* inputs,
                       int* targets) {
  DataLoader dl;
  if (path && path[0] && !dl.load(path)) return 0;
  std::mt19937 rng(seed);
  for (int s = 0; s < steps; ++s)
    dl.get_batch(inputs + (size_t)s * B * T, targets + (size_t)s * B * T, B, T, rng);
  return 1;
}

}  // extern "C"
