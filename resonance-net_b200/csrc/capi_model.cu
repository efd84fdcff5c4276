// C-ABI of the model engine and of the data-parallel plumbing.
#include <sys/stat.h>

#include <chrono>
#include <cstdio>
#include <new>
#include <string>
#include <thread>

#include "dist.h"
#include "engine.h"
#include "status.h"

using rnet_engine::Engine;

struct rnet_model {
  Engine* e = nullptr;
  int* d_in = nullptr;
  int* d_tgt = nullptr;
  float* d_loss = nullptr;
  float* h_loss = nullptr;  // pinned
  int cap = 0;
};

struct rnet_dist {
  rnet_engine::DistComm* c = nullptr;
};

struct rnet_decoder {
  rnet_model* m = nullptr;
  rnet_engine::Decoder d;
};

#define CHECK_M(m)                                                      \
  if (!(m) || !(m)->e) return rnet_status::fail(RNET_ERR_ARG, "null model")

extern "C" {

int rnet_model_create(const rnet_model_config* cfg, int device, int reference_init,
                      rnet_model** out) {
  if (!cfg || !out) return rnet_status::fail(RNET_ERR_ARG, "rnet_model_create: null argument");
  *out = nullptr;
  Engine* e = new (std::nothrow) Engine(*cfg);
  if (!e) return rnet_status::fail(RNET_ERR_ARG, "out of host memory");
  int rc = e->init(device, reference_init != 0);
  if (rc) {
    delete e;
    return rc;
  }
  rnet_model* m = new rnet_model();
  m->e = e;
  *out = m;
  return RNET_OK;
}

int rnet_model_create_from_checkpoint(const char* path, int device, rnet_model** out) {
  if (!path || !out) return rnet_status::fail(RNET_ERR_ARG, "null argument");
  FILE* f = fopen(path, "rb");
  if (!f) return rnet_status::fail(RNET_ERR_IO, std::string("cannot open: ") + path);
  rnet_model_config c;
  const bool ok = fread(&c, sizeof(c), 1, f) == 1;
  fclose(f);
  if (!ok) return rnet_status::fail(RNET_ERR_IO, "checkpoint: truncated header");
  int rc = rnet_model_create(&c, device, 0, out);
  if (rc) return rc;
  rc = (*out)->e->load_weights(path);
  if (rc) {
    rnet_model_destroy(*out);
    *out = nullptr;
  }
  return rc;
}

int rnet_model_destroy(rnet_model* m) {
  if (!m) return RNET_OK;
  if (m->e) cudaStreamSynchronize(m->e->stream());
  cudaFree(m->d_in);
  cudaFree(m->d_tgt);
  cudaFree(m->d_loss);
  cudaFreeHost(m->h_loss);
  delete m->e;
  delete m;
  return RNET_OK;
}

int rnet_model_get_config(const rnet_model* m, rnet_model_config* out) {
  CHECK_M(m);
  if (!out) return rnet_status::fail(RNET_ERR_ARG, "null output");
  *out = m->e->config();
  return RNET_OK;
}

int rnet_model_param_count(const rnet_model* m, size_t* n) {
  CHECK_M(m);
  if (!n) return rnet_status::fail(RNET_ERR_ARG, "null output");
  *n = m->e->param_count();
  return RNET_OK;
}

int rnet_model_device_buffers(rnet_model* m, float** d_params, float** d_grads) {
  CHECK_M(m);
  if (d_params) *d_params = m->e->params();
  if (d_grads) *d_grads = m->e->grads();
  return RNET_OK;
}

int rnet_model_stream(rnet_model* m, void** stream) {
  CHECK_M(m);
  if (!stream) return rnet_status::fail(RNET_ERR_ARG, "null output");
  *stream = (void*)m->e->stream();
  return RNET_OK;
}

int rnet_model_set_params(rnet_model* m, const float* host, size_t n) {
  CHECK_M(m);
  return m->e->set_params_host(host, n);
}
int rnet_model_set_params_device(rnet_model* m, const float* d_params, size_t n) {
  CHECK_M(m);
  if (!d_params) return rnet_status::fail(RNET_ERR_ARG, "null parameter buffer");
  if (n != m->e->param_count())
    return rnet_status::fail(RNET_ERR_ARG, "set_params_device: wrong parameter count");
  RNET_TRY_CUDA(cudaMemcpyAsync(m->e->params(), d_params, n * sizeof(float),
                                cudaMemcpyDeviceToDevice, m->e->stream()));
  int rc = m->e->refresh_shadows();
  if (rc) return rc;
  RNET_TRY_CUDA(cudaStreamSynchronize(m->e->stream()));
  return RNET_OK;
}
int rnet_model_get_params(rnet_model* m, float* host, size_t n) {
  CHECK_M(m);
  return m->e->get_params_host(host, n);
}
int rnet_model_get_grads(rnet_model* m, float* host, size_t n) {
  CHECK_M(m);
  return m->e->get_grads_host(host, n);
}
int rnet_model_params_updated(rnet_model* m) {
  CHECK_M(m);
  return m->e->refresh_shadows();
}
int rnet_model_set_conv_quirk(rnet_model* m, int on) {
  CHECK_M(m);
  m->e->conv_quirk = on != 0;
  return RNET_OK;
}

int rnet_model_set_precision(rnet_model* m, int precision) {
  CHECK_M(m);
  if (precision != 0 && precision != 1)
    return rnet_status::fail(RNET_ERR_ARG, "rnet_model_set_precision: expected 0 (fp32) or 1 (bf16)");
  return m->e->set_precision(precision);
}

int rnet_model_set_optimizer(rnet_model* m, float momentum, float weight_decay,
                             int warmup_steps) {
  CHECK_M(m);
  return m->e->set_optimizer(momentum, weight_decay, warmup_steps);
}

int rnet_model_set_recompute(rnet_model* m, int on) {
  CHECK_M(m);
  return m->e->set_recompute(on != 0);
}

int rnet_model_forward(rnet_model* m, const int* d_tokens, float* d_logits, int batch,
                       int seq_len) {
  CHECK_M(m);
  return m->e->forward(d_tokens, d_logits, batch, seq_len);
}
int rnet_model_backward(rnet_model* m, const float* d_dlogits, const int* d_tokens, int batch,
                        int seq_len) {
  CHECK_M(m);
  return m->e->backward(d_dlogits, d_tokens, batch, seq_len);
}
int rnet_model_zero_grad(rnet_model* m) {
  CHECK_M(m);
  return m->e->zero_grad();
}
int rnet_model_step(rnet_model* m, float lr, float grad_clip) {
  CHECK_M(m);
  return m->e->step(lr, grad_clip);
}
int rnet_model_train_step(rnet_model* m, const int* d_inputs, const int* d_targets, int batch,
                          int seq_len, float lr, float grad_clip, float* d_loss_sum) {
  CHECK_M(m);
  return m->e->train_step(d_inputs, d_targets, batch, seq_len, lr, grad_clip, d_loss_sum);
}

int rnet_model_train_step_host(rnet_model* m, const int* h_inputs, const int* h_targets,
                               int batch, int seq_len, float lr, float grad_clip,
                               float* h_loss_sum) {
  CHECK_M(m);
  if (!h_inputs || !h_targets) return rnet_status::fail(RNET_ERR_ARG, "null token buffer");
  const int N = batch * seq_len;
  if (N <= 0) return rnet_status::fail(RNET_ERR_ARG, "empty batch");
  cudaStream_t s = m->e->stream();
  if (N > m->cap) {
    cudaStreamSynchronize(s);
    cudaFree(m->d_in);
    cudaFree(m->d_tgt);
    m->d_in = m->d_tgt = nullptr;
    RNET_TRY_CUDA(cudaMalloc(&m->d_in, sizeof(int) * N));
    RNET_TRY_CUDA(cudaMalloc(&m->d_tgt, sizeof(int) * N));
    m->cap = N;
  }
  if (!m->d_loss) RNET_TRY_CUDA(cudaMalloc(&m->d_loss, sizeof(float)));
  if (!m->h_loss) RNET_TRY_CUDA(cudaMallocHost(&m->h_loss, sizeof(float)));
  RNET_TRY_CUDA(cudaMemcpyAsync(m->d_in, h_inputs, sizeof(int) * N, cudaMemcpyHostToDevice, s));
  RNET_TRY_CUDA(cudaMemcpyAsync(m->d_tgt, h_targets, sizeof(int) * N, cudaMemcpyHostToDevice, s));
  int rc = m->e->train_step(m->d_in, m->d_tgt, batch, seq_len, lr, grad_clip, m->d_loss);
  if (rc) return rc;
  RNET_TRY_CUDA(cudaMemcpyAsync(m->h_loss, m->d_loss, sizeof(float), cudaMemcpyDeviceToHost, s));
  RNET_TRY_CUDA(cudaStreamSynchronize(s));
  if (h_loss_sum) *h_loss_sum = *m->h_loss;
  return RNET_OK;
}

int rnet_model_topk(rnet_model* m, int layer, const int** d_idx, const float** d_w) {
  CHECK_M(m);
  int* i = nullptr;
  float* w = nullptr;
  int rc = m->e->topk(layer, &i, &w);
  if (rc) return rc;
  if (d_idx) *d_idx = i;
  if (d_w) *d_w = w;
  return RNET_OK;
}

int rnet_model_topk_host(rnet_model* m, int layer, int* h_idx, float* h_w, size_t n) {
  CHECK_M(m);
  int* i = nullptr;
  float* w = nullptr;
  int rc = m->e->topk(layer, &i, &w);
  if (rc) return rc;
  cudaStream_t s = m->e->stream();
  if (h_idx) RNET_TRY_CUDA(cudaMemcpyAsync(h_idx, i, n * sizeof(int), cudaMemcpyDeviceToHost, s));
  if (h_w) RNET_TRY_CUDA(cudaMemcpyAsync(h_w, w, n * sizeof(float), cudaMemcpyDeviceToHost, s));
  RNET_TRY_CUDA(cudaStreamSynchronize(s));
  return RNET_OK;
}

int rnet_model_save(rnet_model* m, const char* path) {
  CHECK_M(m);
  if (!path) return rnet_status::fail(RNET_ERR_ARG, "null path");
  return m->e->save(path);
}
int rnet_model_save_async(rnet_model* m, const char* path) {
  CHECK_M(m);
  if (!path) return rnet_status::fail(RNET_ERR_ARG, "null path");
  return m->e->save_async(path);
}
int rnet_model_save_wait(rnet_model* m) {
  CHECK_M(m);
  return m->e->save_wait();
}
int rnet_model_load_weights(rnet_model* m, const char* path) {
  CHECK_M(m);
  if (!path) return rnet_status::fail(RNET_ERR_ARG, "null path");
  return m->e->load_weights(path);
}

int rnet_model_synchronize(rnet_model* m) {
  CHECK_M(m);
  RNET_TRY_CUDA(cudaStreamSynchronize(m->e->stream()));
  unsigned* d = rnet_status::device_error_word();
  unsigned w = 0;
  if (d) RNET_TRY_CUDA(cudaMemcpy(&w, d, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (w) {
    cudaMemset(d, 0, sizeof(unsigned));
    return rnet_status::fail(RNET_ERR_DEVICE,
                             "device error word set: " + std::to_string(w) +
                                 " (1 = wait timeout, 2 = index out of range, 4 = TMEM)");
  }
  return RNET_OK;
}

int rnet_decoder_create(rnet_model* m, int n_streams, rnet_decoder** out) {
  CHECK_M(m);
  if (!out) return rnet_status::fail(RNET_ERR_ARG, "null output");
  *out = nullptr;
  rnet_decoder* d = new rnet_decoder();
  d->m = m;
  int rc = m->e->decoder_init(&d->d, n_streams);
  if (rc) {
    delete d;
    return rc;
  }
  *out = d;
  return RNET_OK;
}

int rnet_decoder_destroy(rnet_decoder* d) {
  if (!d) return RNET_OK;
  d->m->e->decoder_free(&d->d);
  delete d;
  return RNET_OK;
}

int rnet_decoder_prefill(rnet_decoder* d, const int* d_tokens, int seq_len) {
  if (!d || !d_tokens) return rnet_status::fail(RNET_ERR_ARG, "null argument");
  return d->m->e->prefill(&d->d, d_tokens, seq_len);
}

int rnet_decoder_step(rnet_decoder* d, const int* d_tokens) {
  if (!d) return rnet_status::fail(RNET_ERR_ARG, "null decoder");
  return d->m->e->decode_step(&d->d, d_tokens);
}

int rnet_decoder_set_sampling(rnet_decoder* d, float temperature, float top_p,
                              unsigned long long seed) {
  if (!d) return rnet_status::fail(RNET_ERR_ARG, "null decoder");
  if (!(temperature >= 0.0f) || !(top_p > 0.0f && top_p <= 1.0f))
    return rnet_status::fail(RNET_ERR_ARG,
                             "rnet_decoder_set_sampling: need temperature >= 0, 0 < top_p <= 1");
  if (d->m->e->config().vocab_size > 1024 && temperature > 0.0f)
    return rnet_status::fail(RNET_ERR_UNSUPPORTED, "sampling supports vocab_size <= 1024");
  RNET_TRY_CUDA(cudaStreamSynchronize(d->m->e->stream()));
  d->d.temperature = temperature;
  d->d.top_p = top_p;
  d->d.seed = seed;
  // the captured step has the sampling parameters baked in: capture again
  if (d->d.exec) cudaGraphExecDestroy(d->d.exec);
  if (d->d.graph) cudaGraphDestroy(d->d.graph);
  d->d.exec = nullptr;
  d->d.graph = nullptr;
  return RNET_OK;
}

int rnet_decoder_generate(rnet_decoder* d, int n_steps, int* d_out, int use_graph) {
  if (!d || n_steps < 0) return rnet_status::fail(RNET_ERR_ARG, "bad argument");
  return d->m->e->generate(&d->d, n_steps, d_out, use_graph != 0);
}

int rnet_decoder_outputs(rnet_decoder* d, const float** d_logits, const int** d_next) {
  if (!d) return rnet_status::fail(RNET_ERR_ARG, "null decoder");
  if (d_logits) *d_logits = d->d.logits;
  if (d_next) *d_next = d->d.tok;
  return RNET_OK;
}

int rnet_decoder_outputs_host(rnet_decoder* d, float* h_logits, int* h_next) {
  if (!d) return rnet_status::fail(RNET_ERR_ARG, "null decoder");
  cudaStream_t s = d->m->e->stream();
  const size_t M = d->d.M, V = d->m->e->config().vocab_size;
  if (h_logits)
    RNET_TRY_CUDA(cudaMemcpyAsync(h_logits, d->d.logits, M * V * sizeof(float),
                                  cudaMemcpyDeviceToHost, s));
  if (h_next)
    RNET_TRY_CUDA(cudaMemcpyAsync(h_next, d->d.tok, M * sizeof(int), cudaMemcpyDeviceToHost, s));
  RNET_TRY_CUDA(cudaStreamSynchronize(s));
  return RNET_OK;
}

int rnet_decoder_state(rnet_decoder* d, float** d_state, size_t* floats_per_stream) {
  if (!d) return rnet_status::fail(RNET_ERR_ARG, "null decoder");
  if (d_state) *d_state = d->d.state;
  if (floats_per_stream)
    *floats_per_stream = d->d.floats_per_layer / d->d.M * d->m->e->config().n_layers;
  return RNET_OK;
}

int rnet_model_profile_enable(rnet_model* m, int on) {
  CHECK_M(m);
  m->e->profile_enable(on != 0);
  return RNET_OK;
}

int rnet_model_profile_read(rnet_model* m, double* ms, double* flops, double* bytes,
                            long long* launches, int n_kinds, int reset) {
  CHECK_M(m);
  rnet_engine::ProfStats st;
  int rc = m->e->profile_read(&st, reset != 0);
  if (rc) return rc;
  const int n = n_kinds < rnet_engine::PK_COUNT ? n_kinds : rnet_engine::PK_COUNT;
  for (int i = 0; i < n; ++i) {
    if (ms) ms[i] = st.ms[i];
    if (flops) flops[i] = st.flops[i];
    if (bytes) bytes[i] = st.bytes[i];
    if (launches) launches[i] = st.launches[i];
  }
  return RNET_OK;
}

int rnet_dist_unique_id(unsigned char uid[128]) {
  if (!uid) return rnet_status::fail(RNET_ERR_ARG, "null uid");
  return rnet_engine::dist_unique_id(uid);
}

int rnet_dist_create(int rank, int world, int local_rank, const unsigned char uid[128],
                     int timeout_ms, rnet_dist** out) {
  if (!uid || !out) return rnet_status::fail(RNET_ERR_ARG, "null argument");
  *out = nullptr;
  rnet_engine::DistComm* c = nullptr;
  int rc = rnet_engine::dist_create(rank, world, local_rank, uid, timeout_ms, &c);
  if (rc) return rc;
  *out = new rnet_dist{c};
  return RNET_OK;
}

int rnet_dist_destroy(rnet_dist* d) {
  if (!d) return RNET_OK;
  rnet_engine::dist_destroy(d->c);
  delete d;
  return RNET_OK;
}

int rnet_dist_allreduce_sum(rnet_dist* d, float* d_buf, size_t count, void* stream) {
  if (!d) return RNET_OK;  // inactive: no-op, like the reference
  return rnet_engine::dist_allreduce_on(d->c, d_buf, count, (cudaStream_t)stream);
}

int rnet_dist_group_start(rnet_dist* d) { return d ? rnet_engine::dist_group_start(d->c) : 0; }
int rnet_dist_group_end(rnet_dist* d) { return d ? rnet_engine::dist_group_end(d->c) : 0; }

int rnet_dist_uid_file_write(const char* path, const unsigned char uid[128]) {
  if (!path || !uid) return rnet_status::fail(RNET_ERR_ARG, "null argument");
  const std::string tmp = std::string(path) + ".tmp";
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return rnet_status::fail(RNET_ERR_IO, "cannot write " + tmp);
  const bool ok = fwrite(uid, 1, 128, f) == 128;
  if (fclose(f) != 0 || !ok) return rnet_status::fail(RNET_ERR_IO, "short write " + tmp);
  if (std::rename(tmp.c_str(), path) != 0)
    return rnet_status::fail(RNET_ERR_IO, std::string("rename to ") + path + " failed");
  return RNET_OK;
}

int rnet_dist_uid_file_read(const char* path, int timeout_ms, unsigned char uid[128]) {
  if (!path || !uid) return rnet_status::fail(RNET_ERR_ARG, "null argument");
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    struct stat sb;
    if (stat(path, &sb) == 0 && sb.st_size >= 128) break;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return rnet_status::fail(RNET_ERR_TIMEOUT, std::string("timeout waiting for ") + path);
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
  FILE* f = fopen(path, "rb");
  if (!f) return rnet_status::fail(RNET_ERR_IO, std::string("cannot read ") + path);
  const bool ok = fread(uid, 1, 128, f) == 128;
  fclose(f);
  if (!ok) return rnet_status::fail(RNET_ERR_IO, std::string("short uid file ") + path);
  return RNET_OK;
}

int rnet_model_set_dist(rnet_model* m, rnet_dist* d) {
  CHECK_M(m);
  m->e->dist = d ? d->c : nullptr;
  return RNET_OK;
}

}  // extern "C"
