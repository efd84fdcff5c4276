// Drop-in check: a program written against the reference's C++ API
// (include/layers.h, include/resonance_net.h, include/dist.h) compiled against
// this repository's headers and linked with librnet_b200.so.
//
// Usage: dropin_main <checkpoint_out>
//   trains 3 steps of a tiny model like the reference's train loop
//   (src/main.cpp:126-152), saves, reloads into a fresh model, checks both
//   produce identical logits, and generates 8 tokens. Prints "DROPIN OK".
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "dist.h"
#include "layers.h"
#include "resonance_net.h"

using namespace rnet;

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  DistState dist = dist_init_from_env();
  ModelConfig mcfg;
  mcfg.d_model = 64;
  mcfg.n_layers = 2;
  mcfg.d_ff = 128;
  mcfg.n_slots = 64;
  mcfg.seq_len = 32;
  mcfg.gru_dim = 64;
  TrainConfig tcfg;
  tcfg.batch_size = 2;
  ResonanceNet model;
  if (!model.init(mcfg)) return 1;
  model.set_dist(&dist);
  const int BS = tcfg.batch_size * mcfg.seq_len, V = mcfg.vocab_size;
  int *d_in, *d_tgt;
  float *d_logits, *d_loss, *d_dlogits;
  CUDA_CHECK(cudaMalloc(&d_in, BS * sizeof(int)));
  CUDA_CHECK(cudaMalloc(&d_tgt, BS * sizeof(int)));
  CUDA_CHECK(cudaMalloc(&d_logits, (size_t)BS * V * sizeof(float)));
  CUDA_CHECK(cudaMalloc(&d_dlogits, (size_t)BS * V * sizeof(float)));
  CUDA_CHECK(cudaMalloc(&d_loss, sizeof(float)));
  std::mt19937 rng(42);
  std::vector<int> h_in(BS), h_tgt(BS);
  float first = 0.f, last = 0.f;
  for (int step = 1; step <= 3; ++step) {
    for (int i = 0; i < BS; ++i) {
      h_in[i] = rng() % 256;
      h_tgt[i] = (h_in[i] + 1) % 256;
    }
    CUDA_CHECK(cudaMemcpy(d_in, h_in.data(), BS * sizeof(int), cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(d_tgt, h_tgt.data(), BS * sizeof(int), cudaMemcpyHostToDevice));
    model.zero_grad();
    model.forward(d_in, d_logits, tcfg.batch_size, mcfg.seq_len);
    cross_entropy_forward(d_logits, d_tgt, d_loss, d_dlogits, BS, V, 0);
    scale_grads(d_dlogits, 1.0f / BS, BS * V, 0);
    model.backward(d_dlogits, d_in, tcfg.batch_size, mcfg.seq_len);
    model.step(tcfg, step);
    float h_loss = 0.f;
    CUDA_CHECK(cudaMemcpy(&h_loss, d_loss, sizeof(float), cudaMemcpyDeviceToHost));
    if (step == 1) first = h_loss / BS;
    last = h_loss / BS;
    printf("step %d loss %.5f\n", step, h_loss / BS);
  }
  if (!(std::isfinite(last) && std::fabs(first - std::log(256.0f)) < 0.2f)) {
    printf("unexpected loss\n");
    return 1;
  }
  if (!model.save(argv[1])) return 1;
  ResonanceNet reloaded;
  if (!reloaded.load(argv[1])) return 1;
  if (reloaded.config().d_model != 64 || reloaded.param_count() != model.param_count()) return 1;
  float* d_logits2;
  CUDA_CHECK(cudaMalloc(&d_logits2, (size_t)BS * V * sizeof(float)));
  model.forward(d_in, d_logits, tcfg.batch_size, mcfg.seq_len);
  reloaded.forward(d_in, d_logits2, tcfg.batch_size, mcfg.seq_len);
  CUDA_CHECK(cudaDeviceSynchronize());
  std::vector<float> a((size_t)BS * V), b((size_t)BS * V);
  CUDA_CHECK(cudaMemcpy(a.data(), d_logits, a.size() * 4, cudaMemcpyDeviceToHost));
  CUDA_CHECK(cudaMemcpy(b.data(), d_logits2, b.size() * 4, cudaMemcpyDeviceToHost));
  for (size_t i = 0; i < a.size(); ++i)
    if (a[i] != b[i]) {
      printf("reloaded logits differ at %zu\n", i);
      return 1;
    }
  int prompt[5] = {72, 101, 108, 108, 111};
  int out[8];
  reloaded.generate(prompt, 5, out, 8, 0.0f);
  for (int i = 0; i < 8; ++i)
    if (out[i] < 0 || out[i] >= V) return 1;
  printf("generated:");
  for (int i = 0; i < 8; ++i) printf(" %d", out[i]);
  printf("\nDROPIN OK\n");
  model.destroy();
  reloaded.destroy();
  dist_destroy(dist);
  return 0;
}
