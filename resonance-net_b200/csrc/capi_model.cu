// C-ABI of the model engine and of the data-parallel plumbing.
#include <cstdio>
#include <new>

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

int rnet_model_set_dist(rnet_model* m, rnet_dist* d) {
  CHECK_M(m);
  m->e->dist = d ? d->c : nullptr;
  return RNET_OK;
}

}  // extern "C"
