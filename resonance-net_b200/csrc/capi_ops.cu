// C-ABI of the per-layer operations: one entry per function of the
// reference's include/layers.h:28-153 with the same argument meaning and the
// same overwrite / accumulate contract. Temporaries are stream-ordered
// (cudaMallocAsync / cudaFreeAsync), so no call synchronises the device.
#include <string>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "status.h"

using namespace rnet_gemm;

namespace {

Operand kmaj(const float* p, int ld) { return Operand{p, ld, false}; }
Operand mnmaj(const float* p, int ld) { return Operand{p, ld, true}; }
Epilogue mk(int kind, float* C, int ldc) {
  Epilogue e;
  e.kind = kind;
  e.C = C;
  e.ldc = ldc;
  return e;
}

// Scoped stream-ordered scratch allocation.
struct Tmp {
  cudaStream_t s;
  std::vector<void*> ptrs;
  cudaError_t err = cudaSuccess;
  explicit Tmp(cudaStream_t st) : s(st) {}
  template <class T>
  T* get(size_t n) {
    void* p = nullptr;
    if (err == cudaSuccess) err = cudaMallocAsync(&p, n * sizeof(T) + 16, s);
    if (p) ptrs.push_back(p);
    return static_cast<T*>(p);
  }
  ~Tmp() {
    for (void* p : ptrs) cudaFreeAsync(p, s);
  }
};

#define CK(expr)                                                     \
  do {                                                               \
    cudaError_t _e = (expr);                                         \
    if (_e != cudaSuccess) return rnet_status::fail_cuda(_e, #expr); \
  } while (0)
#define NEED(cond, msg) \
  if (!(cond)) return rnet_status::fail(RNET_ERR_ARG, msg)

unsigned* ew() { return rnet_status::device_error_word(); }

bool a16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

extern "C" {

int rnet_rms_norm_forward(const float* x, const float* w, float* y, float* rms_cache,
                          int batch_seq, int dim, float eps, void* stream) {
  NEED(x && w && y, "rms_norm_forward: null pointer");
  NEED(dim % 4 == 0 && dim <= 2048, "rms_norm_forward: dim must be a multiple of 4, <= 2048");
  NEED(a16(x) && a16(w) && a16(y),
       "rms_norm_forward: x, w and y must be 16-byte aligned (float4 rows)");
  CK(rnet_k::rms_norm_fwd(x, w, y, rms_cache, batch_seq, dim, eps, (cudaStream_t)stream));
  return RNET_OK;
}

int rnet_rms_norm_backward(const float* dy, const float* x, const float* w,
                           const float* rms_cache, float* dx, float* dw, int batch_seq, int dim,
                           void* stream) {
  NEED(dy && x && w && rms_cache && dx && dw, "rms_norm_backward: null pointer");
  NEED(dim % 4 == 0 && dim <= 2048, "rms_norm_backward: dim must be a multiple of 4, <= 2048");
  NEED(a16(dy) && a16(x) && a16(w) && a16(dx),
       "rms_norm_backward: dy, x, w and dx must be 16-byte aligned (bulk-copied rows)");
  CK(rnet_k::rms_norm_bwd(dy, x, w, rms_cache, dx, dw, batch_seq, dim, 0, (cudaStream_t)stream));
  return RNET_OK;
}

int rnet_embed_forward(const int* tokens, const float* table, float* output, int batch_seq,
                       int vocab, int dim, void* stream) {
  NEED(tokens && table && output, "embed_forward: null pointer");
  CK(rnet_k::embed_fwd(tokens, table, output, batch_seq, vocab, dim, ew(), (cudaStream_t)stream));
  return RNET_OK;
}

int rnet_embed_backward(const float* dout, const int* tokens, float* dtable, int batch_seq,
                        int vocab, int dim, void* stream) {
  NEED(dout && tokens && dtable, "embed_backward: null pointer");
  CK(rnet_k::embed_bwd(dout, tokens, dtable, batch_seq, vocab, dim, (cudaStream_t)stream));
  return RNET_OK;
}

int rnet_linear_forward(const float* input, const float* weight, float* output, int M, int N,
                        int K, void* stream) {
  NEED(input && weight && output, "linear_forward: null pointer");
  CK(gemm_tf32x3((cudaStream_t)stream, M, N, K, kmaj(input, K), kmaj(weight, K),
                 mk(EPI_STORE, output, N), 0, 0, ew()));
  return RNET_OK;
}

int rnet_causal_conv_forward(const float* x, float* y, const float* conv3_w,
                             const float* conv7_w, const float* conv15_w, const float* mix_w,
                             float* conv_buf, int batch, int seq_len, int dim, void* stream) {
  NEED(x && y && conv3_w && conv7_w && conv15_w && mix_w && conv_buf,
       "causal_conv_forward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t NE = (size_t)batch * seq_len * dim;
  float* S = conv_buf;
  CK(rnet_k::conv_fwd(x, conv3_w, conv7_w, conv15_w, S, nullptr, conv_buf + NE, conv_buf + 2 * NE,
                      batch, seq_len, dim, s));
  CK(gemm_tf32x3(s, batch * seq_len, dim, dim, kmaj(S, dim), kmaj(mix_w, dim),
                 mk(EPI_STORE, y, dim), 0, 0, ew()));
  return RNET_OK;
}

int rnet_causal_conv_backward(const float* dy, const float* x, const float* conv3_w,
                              const float* conv7_w, const float* conv15_w, const float* mix_w,
                              const float* conv_buf, float* dx, float* d_conv3_w,
                              float* d_conv7_w, float* d_conv15_w, float* d_mix_w, int batch,
                              int seq_len, int dim, int dmix_quirk, void* stream) {
  NEED(dy && x && conv_buf && dx && d_conv3_w && d_conv7_w && d_conv15_w && d_mix_w,
       "causal_conv_backward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch * seq_len;
  const size_t NE = (size_t)N * dim;
  Tmp t(s);
  float* dS = t.get<float>(NE);
  float* Sm = dmix_quirk ? t.get<float>(NE) : nullptr;
  float* parts = t.get<float>(rnet_k::conv_bwd_partials_floats(batch, seq_len, dim));
  CK(t.err);
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(dy, dim), mnmaj(mix_w, dim), mk(EPI_STORE, dS, dim), 0, 0,
                 ew()));
  if (dmix_quirk) CK(rnet_k::add3(conv_buf, conv_buf + NE, conv_buf + 2 * NE, Sm, NE, s));
  CK(gemm_tf32x3(s, dim, dim, N, mnmaj(dy, dim), mnmaj(dmix_quirk ? Sm : conv_buf, dim),
                 mk(EPI_ACCUM, d_mix_w, dim), 0, 0, ew()));
  CK(rnet_k::conv_bwd(dS, x, conv3_w, conv7_w, conv15_w, dx, d_conv3_w, d_conv7_w, d_conv15_w,
                      parts, batch, seq_len, dim, 1, s));
  return RNET_OK;
}

int rnet_min_gru_forward(const float* x, float* y, const float* Wz, const float* Wh,
                         const float* bz, const float* bh, float* z_cache, float* h_cache,
                         int batch, int seq_len, int dim, void* stream) {
  NEED(x && y && Wz && Wh && bz && bh && z_cache && h_cache, "min_gru_forward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch * seq_len;
  Tmp t(s);
  float* P = t.get<float>((size_t)N * 2 * dim);
  CK(t.err);
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(x, dim), kmaj(Wz, dim), mk(EPI_STORE, P, 2 * dim), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(x, dim), kmaj(Wh, dim), mk(EPI_STORE, P + dim, 2 * dim), 0,
                 0, ew()));
  CK(rnet_k::gru_scan_fwd(P, P + dim, 2 * dim, bz, bh, z_cache, h_cache, y, nullptr, nullptr,
                          batch, seq_len, dim, s));
  return RNET_OK;
}

int rnet_min_gru_backward(const float* dy, const float* x, const float* Wz, const float* Wh,
                          const float* bz, const float* bh, const float* z_cache,
                          const float* h_cache, float* dx, float* dWz, float* dWh, float* dbz,
                          float* dbh, int batch, int seq_len, int dim, void* stream) {
  (void)bz;
  NEED(dy && x && Wz && Wh && bh && z_cache && h_cache && dx && dWz && dWh && dbz && dbh,
       "min_gru_backward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch * seq_len;
  Tmp t(s);
  float* ph = t.get<float>((size_t)N * dim);
  float* dzh = t.get<float>((size_t)N * 2 * dim);
  CK(t.err);
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(x, dim), kmaj(Wh, dim), mk(EPI_STORE, ph, dim), 0, 0, ew()));
  CK(rnet_k::gru_scan_bwd(dy, z_cache, h_cache, ph, dim, bh, dzh, dzh + dim, 2 * dim, dbz, dbh,
                          batch, seq_len, dim, s));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(dzh, 2 * dim), mnmaj(Wz, dim), mk(EPI_ACCUM, dx, dim), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(dzh + dim, 2 * dim), mnmaj(Wh, dim), mk(EPI_ACCUM, dx, dim),
                 0, 0, ew()));
  CK(gemm_tf32x3(s, dim, dim, N, mnmaj(dzh, 2 * dim), mnmaj(x, dim), mk(EPI_ACCUM, dWz, dim), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, dim, dim, N, mnmaj(dzh + dim, 2 * dim), mnmaj(x, dim),
                 mk(EPI_ACCUM, dWh, dim), 0, 0, ew()));
  return RNET_OK;
}

int rnet_slot_memory_forward(const float* x, float* y, const float* slot_keys,
                             const float* slot_values, const float* proj_q,
                             const float* proj_out, float* q_cache, float* scores_cache,
                             int* topk_idx_cache, float* topk_w_cache, int batch, int seq_len,
                             int dim, int n_slots, int top_k, void* stream) {
  NEED(x && y && slot_keys && slot_values && proj_q && proj_out && q_cache && topk_idx_cache &&
           topk_w_cache,
       "slot_memory_forward: null pointer");
  NEED(top_k >= 1 && top_k <= 8 && top_k <= n_slots, "slot_memory_forward: top_k must be 1..8");
  NEED(top_k == 2 || scores_cache, "slot_memory_forward: top_k != 2 needs scores_cache");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch * seq_len;
  Tmp t(s);
  float* KT = t.get<float>((size_t)n_slots * dim);
  float* VT = t.get<float>((size_t)n_slots * dim);
  float* r = t.get<float>((size_t)N * dim);
  CK(t.err);
  CK(rnet_k::transpose(slot_keys, KT, dim, n_slots, 0, s));
  CK(rnet_k::transpose(slot_values, VT, dim, n_slots, 0, s));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(x, dim), kmaj(proj_q, dim), mk(EPI_STORE, q_cache, dim), 0,
                 0, ew()));
  if (top_k == 2) {
    Epilogue e = mk(EPI_TOP2, scores_cache, n_slots);
    e.topk_idx = topk_idx_cache;
    e.topk_w = topk_w_cache;
    CK(gemm_tf32x3(s, N, n_slots, dim, kmaj(q_cache, dim), kmaj(KT, dim), e, 0, 0, ew()));
  } else {
    CK(gemm_tf32x3(s, N, n_slots, dim, kmaj(q_cache, dim), kmaj(KT, dim),
                   mk(EPI_STORE, scores_cache, n_slots), 0, 0, ew()));
    CK(rnet_k::topk_rows(scores_cache, topk_idx_cache, topk_w_cache, N, n_slots, top_k, s));
  }
  CK(rnet_k::slot_gather(topk_idx_cache, topk_w_cache, VT, r, N, dim, n_slots, top_k, ew(), s));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(r, dim), kmaj(proj_out, dim), mk(EPI_STORE, y, dim), 0, 0,
                 ew()));
  return RNET_OK;
}

int rnet_slot_memory_backward(const float* dy, const float* x, const float* slot_keys,
                              const float* slot_values, const float* proj_q,
                              const float* proj_out, const float* q_cache,
                              const float* scores_cache, const int* topk_idx_cache,
                              const float* topk_w_cache, float* dx, float* d_slot_keys,
                              float* d_slot_values, float* d_proj_q, float* d_proj_out,
                              int batch, int seq_len, int dim, int n_slots, int top_k,
                              void* stream) {
  (void)scores_cache;  // the cached top-k indices/weights carry everything needed
  NEED(dy && x && slot_keys && slot_values && proj_q && proj_out && q_cache && topk_idx_cache &&
           topk_w_cache && dx && d_slot_keys && d_slot_values && d_proj_q && d_proj_out,
       "slot_memory_backward: null pointer");
  NEED(top_k >= 1 && top_k <= 8, "slot_memory_backward: top_k must be 1..8");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch * seq_len;
  const size_t SD = (size_t)n_slots * dim, ND = (size_t)N * dim;
  Tmp t(s);
  float* KT = t.get<float>(SD);
  float* VT = t.get<float>(SD);
  float* dKT = t.get<float>(SD);
  float* dVT = t.get<float>(SD);
  float* r = t.get<float>(ND);
  float* dr = t.get<float>(ND);
  float* dq = t.get<float>(ND);
  CK(t.err);
  CK(rnet_k::transpose(slot_keys, KT, dim, n_slots, 0, s));
  CK(rnet_k::transpose(slot_values, VT, dim, n_slots, 0, s));
  CK(cudaMemsetAsync(dKT, 0, SD * sizeof(float), s));
  CK(cudaMemsetAsync(dVT, 0, SD * sizeof(float), s));
  CK(rnet_k::slot_gather(topk_idx_cache, topk_w_cache, VT, r, N, dim, n_slots, top_k, ew(), s));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(dy, dim), mnmaj(proj_out, dim), mk(EPI_STORE, dr, dim), 0,
                 0, ew()));
  CK(gemm_tf32x3(s, dim, dim, N, mnmaj(dy, dim), mnmaj(r, dim), mk(EPI_ACCUM, d_proj_out, dim), 0,
                 0, ew()));
  CK(rnet_k::slot_sparse_bwd(dr, topk_idx_cache, topk_w_cache, VT, KT, q_cache, dq, dVT, dKT, N,
                             dim, n_slots, top_k, ew(), s));
  CK(rnet_k::transpose(dKT, d_slot_keys, n_slots, dim, 1, s));
  CK(rnet_k::transpose(dVT, d_slot_values, n_slots, dim, 1, s));
  CK(gemm_tf32x3(s, N, dim, dim, kmaj(dq, dim), mnmaj(proj_q, dim), mk(EPI_ACCUM, dx, dim), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, dim, dim, N, mnmaj(dq, dim), mnmaj(x, dim), mk(EPI_ACCUM, d_proj_q, dim), 0, 0,
                 ew()));
  return RNET_OK;
}

int rnet_swiglu_forward(const float* x, float* y, const float* gate_w, const float* up_w,
                        const float* down_w, float* gate_cache, float* up_cache, int batch_seq,
                        int dim, int d_ff, void* stream) {
  NEED(x && y && gate_w && up_w && down_w && gate_cache && up_cache,
       "swiglu_forward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch_seq;
  Tmp t(s);
  float* H = t.get<float>((size_t)N * d_ff);
  CK(t.err);
  if (up_w == gate_w + (size_t)d_ff * dim && d_ff % 64 == 0) {
    Epilogue e;
    e.kind = EPI_SWIGLU_FWD;
    e.G = gate_cache;
    e.U = up_cache;
    e.H = H;
    e.ldf = d_ff;
    CK(gemm_tf32x3(s, N, d_ff, dim, kmaj(x, dim), kmaj(gate_w, dim), e, d_ff, 0, ew()));
  } else {
    CK(gemm_tf32x3(s, N, d_ff, dim, kmaj(x, dim), kmaj(gate_w, dim),
                   mk(EPI_STORE, gate_cache, d_ff), 0, 0, ew()));
    CK(gemm_tf32x3(s, N, d_ff, dim, kmaj(x, dim), kmaj(up_w, dim), mk(EPI_STORE, up_cache, d_ff),
                   0, 0, ew()));
    CK(rnet_k::silu_mul(gate_cache, up_cache, H, (size_t)N * d_ff, s));
  }
  CK(gemm_tf32x3(s, N, dim, d_ff, kmaj(H, d_ff), kmaj(down_w, d_ff), mk(EPI_STORE, y, dim), 0, 0,
                 ew()));
  return RNET_OK;
}

int rnet_swiglu_backward(const float* dy, const float* x, const float* gate_w,
                         const float* up_w, const float* down_w, const float* gate_cache,
                         const float* up_cache, float* dx, float* d_gate_w, float* d_up_w,
                         float* d_down_w, int batch_seq, int dim, int d_ff, void* stream) {
  NEED(dy && x && gate_w && up_w && down_w && gate_cache && up_cache && dx && d_gate_w &&
           d_up_w && d_down_w,
       "swiglu_backward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const int N = batch_seq, F = d_ff;
  Tmp t(s);
  float* H = t.get<float>((size_t)N * F);
  float* dGU = t.get<float>((size_t)N * 2 * F);
  CK(t.err);
  CK(rnet_k::silu_mul(gate_cache, up_cache, H, (size_t)N * F, s));
  CK(gemm_tf32x3(s, N, F, dim, kmaj(dy, dim), mnmaj(down_w, F), mk(EPI_STORE, dGU, 2 * F), 0, 0,
                 ew()));
  CK(rnet_k::swiglu_bwd_pointwise(dGU, 2 * F, gate_cache, up_cache, N, F, s));
  CK(gemm_tf32x3(s, dim, F, N, mnmaj(dy, dim), mnmaj(H, F), mk(EPI_ACCUM, d_down_w, F), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, N, dim, F, kmaj(dGU, 2 * F), mnmaj(gate_w, dim), mk(EPI_ACCUM, dx, dim), 0, 0,
                 ew()));
  CK(gemm_tf32x3(s, N, dim, F, kmaj(dGU + F, 2 * F), mnmaj(up_w, dim), mk(EPI_ACCUM, dx, dim), 0,
                 0, ew()));
  CK(gemm_tf32x3(s, F, dim, N, mnmaj(dGU, 2 * F), mnmaj(x, dim), mk(EPI_ACCUM, d_gate_w, dim), 0,
                 0, ew()));
  CK(gemm_tf32x3(s, F, dim, N, mnmaj(dGU + F, 2 * F), mnmaj(x, dim), mk(EPI_ACCUM, d_up_w, dim), 0,
                 0, ew()));
  return RNET_OK;
}

int rnet_cross_entropy_forward(const float* logits, const int* targets, float* loss,
                               float* dlogits, int batch_seq, int vocab, void* stream) {
  NEED(logits && targets && loss && dlogits, "cross_entropy_forward: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  Tmp t(s);
  float* parts = t.get<float>(rnet_k::ce_partials_floats(batch_seq));
  CK(t.err);
  CK(rnet_k::cross_entropy(logits, targets, loss, dlogits, 1.0f, parts, batch_seq, vocab, ew(), s));
  return RNET_OK;
}

int rnet_residual_add(float* x, const float* y, size_t n, void* stream) {
  NEED(x && y, "residual_add: null pointer");
  CK(rnet_k::residual_add(x, y, n, (cudaStream_t)stream));
  return RNET_OK;
}

int rnet_scale_grads(float* grads, float scale, size_t n, void* stream) {
  NEED(grads, "scale_grads: null pointer");
  CK(rnet_k::scale(grads, scale, n, (cudaStream_t)stream));
  return RNET_OK;
}

}  // extern "C"
