// ResonanceNet model engine (see engine.h).
//
// Reference orchestration: src/resonance_net.cpp:44-216 (allocation, init),
// :218-343 (forward with caches), :346-408 (inference forward), :411-548
// (backward), :551-697 (step, zero_grad), :743-824 (checkpoint).
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "dist.h"
#include "engine.h"
#include "gemm.cuh"
#include "kernels.cuh"
#include "status.h"

namespace rnet_engine {
using rnet_gemm::Epilogue;
using rnet_gemm::Operand;
using namespace rnet_gemm;

namespace {

Operand kmaj(const float* p, int ld) { return Operand{p, ld, false}; }
Operand mnmaj(const float* p, int ld) { return Operand{p, ld, true}; }
// fp32 operand, or its bf16 copy when `bf` (same shape and pitch)
Operand kop(bool bf, const float* p, const __nv_bfloat16* h, int ld) {
  return bf ? bf16_operand(h, ld, false) : kmaj(p, ld);
}
Operand mop(bool bf, const float* p, const __nv_bfloat16* h, int ld) {
  return bf ? bf16_operand(h, ld, true) : mnmaj(p, ld);
}

Epilogue epi_store(float* C, int ldc) {
  Epilogue e;
  e.kind = EPI_STORE;
  e.C = C;
  e.ldc = ldc;
  return e;
}
Epilogue epi_accum(float* C, int ldc) {
  Epilogue e;
  e.kind = EPI_ACCUM;
  e.C = C;
  e.ldc = ldc;
  return e;
}

size_t layer_count(const rnet_model_config& c) {
  const size_t D = c.d_model, F = c.d_ff, S = c.n_slots;
  return 4 * D + 25 * D + 3 * D * D + 2 * D + 2 * D * S + 2 * D * D + 3 * D * F;
}

}  // namespace

#define CK(expr)                                                     \
  do {                                                               \
    cudaError_t _e = (expr);                                         \
    if (_e != cudaSuccess) return rnet_status::fail_cuda(_e, #expr); \
  } while (0)

Engine::Engine(const rnet_model_config& c) : cfg_(c) {}

Engine::~Engine() {
  if (device_ >= 0) cudaSetDevice(device_);
  save_wait();
  if (train_exec_) cudaGraphExecDestroy(train_exec_);
  cudaFree(g_in_);
  cudaFree(g_tgt_);
  cudaFree(snap_);
  if (snap_host_) cudaFreeHost(snap_host_);
  if (snap_ready_) cudaEventDestroy(snap_ready_);
  if (host_ready_) cudaEventDestroy(host_ready_);
  if (save_stream_) cudaStreamDestroy(save_stream_);
  if (stream_) cudaStreamSynchronize(stream_);
  cudaFree(params_);
  cudaFree(grads_);
  cudaFree(KT_);
  cudaFree(VT_);
  cudaFree(params16_);
  cudaFree(KT16_);
  cudaFree(velocity_);
  cudaFree(comm16_);
  cudaFree(dKV_);
  for (cudaEvent_t e : ev_pool_) cudaEventDestroy(e);
  cudaFree(scratch_);
  cudaFree(arena_);
  if (ev_fork_) cudaEventDestroy(ev_fork_);
  if (ev_join_) cudaEventDestroy(ev_join_);
  if (wstream_) cudaStreamDestroy(wstream_);
  if (stream_) cudaStreamDestroy(stream_);
}

int Engine::gemm_err(cudaError_t e, const char* what) {
  return rnet_status::fail_cuda(e, what);
}

int Engine::init(int device, bool reference_init) {
  const rnet_model_config& c = cfg_;
  if (c.d_model <= 0 || c.n_layers <= 0 || c.d_ff <= 0 || c.n_slots <= 0 || c.vocab_size <= 0)
    return rnet_status::fail(RNET_ERR_ARG, "model config: non-positive dimension");
  if (c.d_model % 32 || c.d_ff % 32 || c.n_slots % 4 || c.vocab_size % 4)
    return rnet_status::fail(RNET_ERR_ARG,
                             "model config: d_model and d_ff must be multiples of 32, "
                             "n_slots and vocab_size multiples of 4");
  if (c.d_model > 2048) return rnet_status::fail(RNET_ERR_UNSUPPORTED, "d_model > 2048");
  if (c.vocab_size > 1024) return rnet_status::fail(RNET_ERR_UNSUPPORTED, "vocab_size > 1024");
  if (c.slot_top_k < 1 || c.slot_top_k > 8 || c.slot_top_k > c.n_slots)
    return rnet_status::fail(RNET_ERR_ARG, "slot_top_k must be in [1, min(8, n_slots)]");
  device_ = device;
  CK(cudaSetDevice(device));
  CK(cudaStreamCreate(&stream_));  // blocking w.r.t. the legacy stream, like the reference
  CK(cudaStreamCreateWithFlags(&wstream_, cudaStreamNonBlocking));
  if (const char* v = getenv("RNET_TRAIN_GRAPH")) train_graphs_ = v[0] != '0';
  CK(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming));

  const size_t D = c.d_model, V = c.vocab_size, F = c.d_ff, S = c.n_slots, L = c.n_layers;
  P_ = 2 * V * D + D + L * layer_count(c);
  CK(cudaMalloc(&params_, P_ * sizeof(float)));
  CK(cudaMalloc(&grads_, P_ * sizeof(float)));
  CK(cudaMemset(grads_, 0, P_ * sizeof(float)));
  auto bind = [&](float* base, std::vector<LayerParams>& out, float** e, float** o, float** f) {
    float* p = base;
    auto take = [&](size_t n) { float* r = p; p += n; return r; };
    *e = take(V * D);
    *o = take(V * D);
    *f = take(D);
    out.resize(L);
    for (size_t l = 0; l < L; ++l) {
      LayerParams& q = out[l];
      q.offset = (size_t)(p - base);
      q.n1 = take(D); q.n2 = take(D); q.n3 = take(D); q.n4 = take(D);
      q.c3 = take(3 * D); q.c7 = take(7 * D); q.c15 = take(15 * D); q.mix = take(D * D);
      q.Wz = take(D * D); q.Wh = take(D * D); q.bz = take(D); q.bh = take(D);
      q.keys = take(D * S); q.vals = take(D * S); q.pq = take(D * D); q.pout = take(D * D);
      q.gate = take(F * D); q.up = take(F * D); q.down = take(D * F);
      q.count = (size_t)(p - base) - q.offset;
    }
  };
  bind(params_, W_, &embed_, &outw_, &fnorm_);
  bind(grads_, G_, &g_embed_, &g_outw_, &g_fnorm_);
  CK(cudaMalloc(&KT_, L * S * D * sizeof(float)));
  CK(cudaMalloc(&VT_, L * S * D * sizeof(float)));
  // key / value scatter gradients, per layer [keys | values] of [S, D] each
  CK(cudaMalloc(&dKV_, 2 * L * S * D * sizeof(float)));
  const size_t scr = rnet_k::sgd_scratch_floats() + 64;
  CK(cudaMalloc(&scratch_, scr * sizeof(float)));
  loss_dev_ = scratch_ + rnet_k::sgd_scratch_floats();
  norm_dev_ = loss_dev_ + 1;

  if (reference_init) {
    // Same distributions, seeds and tensor order as the reference
    // (src/resonance_net.cpp:27-42 and :180-216): U(-1/sqrt(fan_in), +1/sqrt(fan_in))
    // from std::mt19937(seed), seed = 42, 43, ... in tensor order; norm gains 1,
    // biases 0.
    std::vector<float> h(P_, 0.0f);
    unsigned seed = 42;
    auto xavier = [&](float* dptr, size_t n, int fan_in) {
      std::mt19937 rng(seed++);
      const float sc = 1.0f / sqrtf((float)fan_in);
      std::uniform_real_distribution<float> dist(-sc, sc);
      float* hp = h.data() + (dptr - params_);
      for (size_t i = 0; i < n; ++i) hp[i] = dist(rng);
    };
    auto ones = [&](float* dptr, size_t n) {
      float* hp = h.data() + (dptr - params_);
      for (size_t i = 0; i < n; ++i) hp[i] = 1.0f;
    };
    xavier(embed_, V * D, (int)D);
    xavier(outw_, V * D, (int)D);
    ones(fnorm_, D);
    for (size_t l = 0; l < L; ++l) {
      LayerParams& w = W_[l];
      ones(w.n1, D); ones(w.n2, D); ones(w.n3, D); ones(w.n4, D);
      xavier(w.c3, 3 * D, (int)D);
      xavier(w.c7, 7 * D, (int)D);
      xavier(w.c15, 15 * D, (int)D);
      xavier(w.mix, D * D, (int)D);
      xavier(w.Wz, D * D, (int)D);
      xavier(w.Wh, D * D, (int)D);
      xavier(w.keys, D * S, (int)D);
      xavier(w.vals, D * S, (int)D);
      xavier(w.pq, D * D, (int)D);
      xavier(w.pout, D * D, (int)D);
      xavier(w.gate, D * F, (int)D);
      xavier(w.up, D * F, (int)D);
      xavier(w.down, F * D, (int)F);
    }
    CK(cudaMemcpy(params_, h.data(), P_ * sizeof(float), cudaMemcpyHostToDevice));
  } else {
    CK(cudaMemset(params_, 0, P_ * sizeof(float)));
  }
  return refresh_shadows();
}

int Engine::set_precision(int p) {
  if (p != 0 && p != 1) return rnet_status::fail(RNET_ERR_ARG, "precision must be 0 or 1");
  if (p == 1 && !params16_) {
    const size_t KT = (size_t)cfg_.n_layers * cfg_.n_slots * cfg_.d_model;
    CK(cudaMalloc(&params16_, P_ * sizeof(__nv_bfloat16)));
    CK(cudaMalloc(&KT16_, KT * sizeof(__nv_bfloat16)));
  }
  precision = p;
  return refresh_shadows();
}

int Engine::refresh_shadows() { return refresh_shadows_impl(false); }

// Transposed key / value copies (and, in bf16 mode, the bf16 shadows of the
// parameters — unless the SGD update has just written them — and of the
// transposed keys) after a weight change.
int Engine::refresh_shadows_impl(bool params16_current) {
  const int D = cfg_.d_model, S = cfg_.n_slots, L = cfg_.n_layers;
  // keys / values of all layers in one launch (keys and values are adjacent
  // in a layer's parameter range; layers are evenly spaced)
  const size_t kv = (size_t)(W_[0].vals - W_[0].keys);
  const size_t layer = L > 1 ? (size_t)(W_[1].keys - W_[0].keys) : 0;
  for (int l = 1; l < L; ++l)
    if ((size_t)(W_[l].keys - W_[0].keys) != l * layer || (size_t)(W_[l].vals - W_[l].keys) != kv)
      return rnet_status::fail(RNET_ERR_ARG, "refresh_shadows: unexpected parameter layout");
  CK(rnet_k::transpose_pairs(W_[0].keys, kv, layer, KT_, VT_, (size_t)S * D, L, D, S, 0,
                             stream_));
  if (precision == 1) {
    if (!params16_current) CK(rnet_k::to_bf16(params_, params16_, P_, stream_));
    CK(rnet_k::to_bf16(KT_, KT16_, (size_t)L * S * D, stream_));
  }
  return RNET_OK;
}

int Engine::set_params_host(const float* h, size_t n) {
  if (n != P_) return rnet_status::fail(RNET_ERR_ARG, "set_params: wrong parameter count");
  CK(cudaMemcpyAsync(params_, h, P_ * sizeof(float), cudaMemcpyHostToDevice, stream_));
  int rc = refresh_shadows();
  if (rc) return rc;
  CK(cudaStreamSynchronize(stream_));
  return RNET_OK;
}

int Engine::get_params_host(float* h, size_t n) {
  if (n != P_) return rnet_status::fail(RNET_ERR_ARG, "get_params: wrong parameter count");
  CK(cudaMemcpyAsync(h, params_, P_ * sizeof(float), cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  return RNET_OK;
}

int Engine::get_grads_host(float* h, size_t n) {
  if (n != P_) return rnet_status::fail(RNET_ERR_ARG, "get_grads: wrong parameter count");
  CK(cudaMemcpyAsync(h, grads_, P_ * sizeof(float), cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  return RNET_OK;
}

int Engine::ensure_capacity(int N, bool with_caches) {
  const bool bf = precision == 1;
  if (N <= cap_N_ && (cap_caches_ || !with_caches) && (cap_bf16_ || !bf) &&
      cap_recompute_ == recompute_)
    return RNET_OK;
  const size_t D = cfg_.d_model, F = cfg_.d_ff, S = cfg_.n_slots, V = cfg_.vocab_size;
  const size_t L = cfg_.n_layers, k = cfg_.slot_top_k;
  const size_t n = (size_t)N;
  const size_t nact = with_caches && !recompute_ ? L : 1;
  std::vector<std::pair<void**, size_t>> plan;  // (slot, bytes)
  act_.assign(nact, LayerAct{});
  auto f = [&](float** p, size_t cnt) { plan.push_back({(void**)p, cnt * sizeof(float)}); };
  auto hb = [&](__nv_bfloat16** p, size_t cnt) {
    if (bf) plan.push_back({(void**)p, cnt * sizeof(__nv_bfloat16)});
    else *p = nullptr;
  };
  for (size_t l = 0; l < nact; ++l) {
    LayerAct& a = act_[l];
    f(&a.n1, n * D); f(&a.n2, n * D); f(&a.n3, n * D); f(&a.n4, n * D);
    f(&a.rinv1, n); f(&a.rinv2, n); f(&a.rinv3, n); f(&a.rinv4, n);
    f(&a.S, n * D); f(&a.Sq, n * D); f(&a.P, 2 * n * D); f(&a.z, n * D); f(&a.h, n * D);
    f(&a.q, n * D); f(&a.r, n * D);
    plan.push_back({(void**)&a.idx, n * k * sizeof(int)});
    f(&a.w, n * k);
    f(&a.r1, n * D); f(&a.r2, n * D); f(&a.r3, n * D);
    f(&a.G, n * F); f(&a.U, n * F); f(&a.H, n * F);
    hb(&a.n2h, n * D); hb(&a.n3h, n * D); hb(&a.n4h, n * D); hb(&a.Sh, n * D);
    hb(&a.Sqh, n * D); hb(&a.qh, n * D); hb(&a.rh, n * D); hb(&a.Hh, n * F);
  }
  hb(&nfh_, n * D);
  f(&X_, (with_caches ? (L + 1) : 2) * n * D);
  f(&nf_, n * D);
  f(&rinvf_, n);
  f(&logits_, n * V);
  f(&dlogits_, n * V);
  if (k != 2) f(&scores_, n * S);
  else scores_ = nullptr;
  if (with_caches) {
    f(&dX_, n * D); f(&dsub_, n * D); f(&dS_, n * D); f(&dq_, n * D); f(&dr_, n * D);
    f(&dPZH_, 2 * n * D); f(&dGU_, 2 * n * F); f(&dnf_, n * D);
    // conv weight-grad partials and CE loss partials share it
    const size_t cp = rnet_k::conv_bwd_partials_floats(N, 1, D),
                 cep = rnet_k::ce_partials_floats(N) + 8;
    f(&conv_parts_, cp > cep ? cp : cep);
    hb(&dlogitsh_, n * V); hb(&dXh_, n * D); hb(&dGUh_, 2 * n * F); hb(&dqh_, n * D);
    hb(&dPZHh_, 2 * n * D);
  } else {
    dlogitsh_ = dXh_ = dGUh_ = dqh_ = dPZHh_ = nullptr;
    dX_ = dsub_ = dS_ = dq_ = dr_ = dPZH_ = dGU_ = dnf_ = conv_parts_ = nullptr;
  }
  size_t total = 0;
  for (auto& e : plan) total += (e.second + 255) & ~size_t(255);
  if (arena_) {
    cudaStreamSynchronize(stream_);
    cudaFree(arena_);
    arena_ = nullptr;
  }
  CK(cudaMalloc(&arena_, total));
  arena_bytes_ = total;
  char* p = (char*)arena_;
  for (auto& e : plan) {
    *e.first = p;
    p += (e.second + 255) & ~size_t(255);
  }
  cap_N_ = N;
  cap_caches_ = with_caches;
  cap_bf16_ = bf;
  cap_recompute_ = recompute_;
  have_cache_ = false;
  return RNET_OK;
}

// ------------------------------------------------------------------ profiling
cudaEvent_t Engine::prof_event() {
  if (ev_used_ == ev_pool_.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    ev_pool_.push_back(e);
  }
  return ev_pool_[ev_used_++];
}

void Engine::prof_begin(cudaEvent_t* a) {
  *a = prof_event();
  cudaEventRecord(*a, stream_);
}

void Engine::prof_end(cudaEvent_t a, int kind, double flops, double bytes) {
  cudaEvent_t b = prof_event();
  cudaEventRecord(b, stream_);
  prof_.push_back(ProfRec{kind, flops, bytes, a, b});
}

int Engine::profile_read(ProfStats* out, bool reset) {
  CK(cudaStreamSynchronize(stream_));
  std::memset(out, 0, sizeof(*out));
  for (const ProfRec& r : prof_) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, r.a, r.b));
    out->ms[r.kind] += ms;
    out->flops[r.kind] += r.flops;
    out->bytes[r.kind] += r.bytes;
    out->launches[r.kind] += 1;
  }
  if (reset) {
    prof_.clear();
    ev_used_ = 0;
  }
  return RNET_OK;
}

// Time one launch group of a kernel class when profiling is on.
#define PROF(kind, flops, bytes, expr)                    \
  do {                                                    \
    cudaEvent_t _pa = nullptr;                            \
    if (prof_on_) prof_begin(&_pa);                       \
    CK(expr);                                             \
    if (prof_on_) prof_end(_pa, (kind), (flops), (bytes)); \
  } while (0)

// GEMM through the engine: algorithmic FLOPs 2MNK, bytes = operands + output
// (+ output read for residual / accumulate epilogues).
#define MMS(M, N, K, A, B, E, PAIR, SPLITS)                                               \
  PROF(PK_GEMM, 2.0 * (M) * (N) * (K),                                                    \
       4.0 * ((double)(M) * (K) + (double)(N) * (K) +                                     \
              (double)(M) * (N) * (((E).kind == EPI_RESID || (E).kind == EPI_ACCUM) ? 2 : 1)), \
       gemm_tf32x3(stream_, (M), (N), (K), (A), (B), (E), (PAIR), (SPLITS), err, precision))
#define MM(M, N, K, A, B, E, PAIR) MMS(M, N, K, A, B, E, PAIR, 0)
// Weight-gradient GEMM of the backward on the side stream (after fork()):
// it runs beside the data-gradient work of the same sublayer, so one GEMM's
// last partial wave fills SMs the other leaves idle. Profiled runs keep it on
// the main stream so the per-class event timing stays exact.
#define MM_W(M, N, K, A, B, E)                                                    \
  do {                                                                            \
    if (prof_on_) {                                                               \
      MM(M, N, K, A, B, E, 0);                                                    \
    } else {                                                                      \
      CK(gemm_tf32x3(wstream_, (M), (N), (K), (A), (B), (E), 0, 0, err, precision)); \
    }                                                                             \
  } while (0)
// residual accumulation: one K pass (deterministic, one rounding per element)
#define MM_RES(M, N, K, A, B, C) MMS(M, N, K, A, B, epi_accum(C, N), 0, 1)

// ------------------------------------------------------------------ forward
int Engine::layer_forward(int l, const float* Xl, float* Xn, LayerAct& a, int B, int T,
                          bool train) {
  const int N = B * T, D = cfg_.d_model, F = cfg_.d_ff, S = cfg_.n_slots, k = cfg_.slot_top_k;
  const float eps = cfg_.rms_eps;
  const LayerParams& w = W_[l];
  unsigned* err = rnet_status::device_error_word();
  cudaStream_t s = stream_;
  const float* KT = KT_ + (size_t)l * S * D;
  const float* VT = VT_ + (size_t)l * S * D;
  const double ND4 = 4.0 * N * D;
  const bool bf = precision == 1;
  // 1. multi-scale causal conv (reference layer_forward :287-299)
  // Residual sums are seeded by the kernel that already holds the residual
  // row (RMSNorm input copy, scan second output) and the GEMM accumulates
  // into them (red.add: the same single rounding as R + acc, without the
  // epilogue's dependent residual loads).
  PROF(PK_RMS_FWD, 0, 3 * ND4, rnet_k::rms_norm_fwd(Xl, w.n1, a.n1, a.rinv1, N, D, eps, s, a.r1));
  // bf16 mode: S (and the dmix operand Sq) only as the bf16 copies the
  // GEMMs read; the fp32 ones would never be read
  const double ND2 = 2.0 * N * D;
  if (bf)
    PROF(PK_CONV_FWD, 50.0 * N * D, ND4 + (train && conv_quirk ? 2 : 1) * ND2,
         rnet_k::conv_fwd_bf16(a.n1, w.c3, w.c7, w.c15, a.Sh, train && conv_quirk ? a.Sqh : nullptr,
                               B, T, D, s));
  else
    PROF(PK_CONV_FWD, 50.0 * N * D, (conv_quirk ? 3 : 2) * ND4,
         rnet_k::conv_fwd(a.n1, w.c3, w.c7, w.c15, a.S, conv_quirk ? a.Sq : nullptr, nullptr,
                          nullptr, B, T, D, s));
  MM_RES(N, D, D, kop(bf, a.S, a.Sh, D), kop(bf, w.mix, bf ? h16(w.mix) : nullptr, D), a.r1);
  // 2. MinGRU (:301-313): P = n2 [Wz;Wh]^T, fused gate + scan + residual
  PROF(PK_RMS_FWD, 0, ND4 + (bf ? ND2 : ND4),
       rnet_k::rms_norm_fwd(a.r1, w.n2, bf ? nullptr : a.n2, a.rinv2, N, D, eps, s, nullptr,
                            a.n2h));
  MM(N, 2 * D, D, kop(bf, a.n2, a.n2h, D), kop(bf, w.Wz, bf ? h16(w.Wz) : nullptr, D),
     epi_store(a.P, 2 * D), 0);
  // training keeps e = h~ - h_prev (all the backward needs), prefill keeps h
  PROF(PK_SCAN_FWD, 0, 7 * ND4,
       rnet_k::gru_scan_fwd(a.P, a.P + D, 2 * D, w.bz, w.bh, a.z, a.h, nullptr, a.r1, a.r2, B, T,
                            D, s, train, a.r3));
  // 3. slot memory (:315-330)
  PROF(PK_RMS_FWD, 0, ND4 + (bf ? ND2 : ND4),
       rnet_k::rms_norm_fwd(a.r2, w.n3, bf ? nullptr : a.n3, a.rinv3, N, D, eps, s, nullptr,
                            a.n3h));
  {
    Epilogue e = epi_store(a.q, D);
    e.C16 = bf ? a.qh : nullptr;
    MM(N, D, D, kop(bf, a.n3, a.n3h, D), kop(bf, w.pq, bf ? h16(w.pq) : nullptr, D), e, 0);
  }
  if (k == 2) {
    Epilogue e;
    e.kind = EPI_TOP2;
    e.topk_idx = a.idx;
    e.topk_w = a.w;
    MM(N, S, D, kop(bf, a.q, a.qh, D),
       kop(bf, KT, bf ? KT16_ + (size_t)l * S * D : nullptr, D), e, 0);
  } else {
    MM(N, S, D, kmaj(a.q, D), kmaj(KT, D), epi_store(scores_, S), 0);
    PROF(PK_OTHER, 0, 4.0 * N * S, rnet_k::topk_rows(scores_, a.idx, a.w, N, S, k, s));
  }
  PROF(PK_SLOT_GATHER, 2.0 * k * N * D, k * ND4 + (bf ? ND2 : ND4),
       rnet_k::slot_gather(a.idx, a.w, VT, bf ? nullptr : a.r, N, D, S, k, err, s, a.rh));
  MM_RES(N, D, D, kop(bf, a.r, a.rh, D), kop(bf, w.pout, bf ? h16(w.pout) : nullptr, D), a.r3);
  // 4. SwiGLU FFN (:332-342): paired gate|up tiles, SiLU*up in the epilogue
  PROF(PK_RMS_FWD, 0, 2 * ND4 + (bf ? ND2 : ND4),
       rnet_k::rms_norm_fwd(a.r3, w.n4, bf ? nullptr : a.n4, a.rinv4, N, D, eps, s, Xn, a.n4h));
  {
    Epilogue e;
    e.kind = EPI_SWIGLU_FWD;
    e.G = a.G;
    e.U = a.U;
    e.H = bf ? nullptr : a.H;  // bf16 mode: H only as the bf16 copy
    e.H16 = bf ? a.Hh : nullptr;
    e.ldf = F;
    MM(N, F, D, kop(bf, a.n4, a.n4h, D), kop(bf, w.gate, bf ? h16(w.gate) : nullptr, D), e,
       F);  // 2*N*F*D each for gate and up
    if (prof_on_) prof_.back().flops *= 2.0;
  }
  MM_RES(N, D, F, kop(bf, a.H, a.Hh, F), kop(bf, w.down, bf ? h16(w.down) : nullptr, F), Xn);
  return RNET_OK;
}

int Engine::forward(const int* d_tokens, float* d_logits, int B, int T) {
  if (B <= 0 || T <= 0) return rnet_status::fail(RNET_ERR_ARG, "forward: empty batch");
  const int N = B * T, D = cfg_.d_model, V = cfg_.vocab_size;
  // Same cache rule as the reference (src/resonance_net.cpp:245).
  const bool caches = N <= 64 * (cfg_.seq_len > 0 ? cfg_.seq_len : 256);
  int rc = ensure_capacity(N, caches);
  if (rc) return rc;
  cudaStream_t s = stream_;
  unsigned* err = rnet_status::device_error_word();
  const size_t ND = (size_t)N * D;
  PROF(PK_EMBED, 0, 4.0 * ND, rnet_k::embed_fwd(d_tokens, embed_, X_, N, V, D, err, s));
  for (int l = 0; l < cfg_.n_layers; ++l) {
    const float* Xl = caches ? X_ + (size_t)l * ND : X_ + (size_t)(l & 1) * ND;
    float* Xn = caches ? X_ + (size_t)(l + 1) * ND : X_ + (size_t)((l + 1) & 1) * ND;
    rc = layer_forward(l, Xl, Xn, caches && !recompute_ ? act_[l] : act_[0], B, T, caches);
    if (rc) return rc;
  }
  const float* XL = caches ? X_ + (size_t)cfg_.n_layers * ND : X_ + (size_t)(cfg_.n_layers & 1) * ND;
  const bool bf = precision == 1;
  PROF(PK_RMS_FWD, 0, (bf ? 6.0 : 8.0) * ND,
       rnet_k::rms_norm_fwd(XL, fnorm_, bf ? nullptr : nf_, rinvf_, N, D, cfg_.rms_eps, s, nullptr,
                            nfh_));
  MM(N, V, D, kop(bf, nf_, nfh_, D), kop(bf, outw_, bf ? h16(outw_) : nullptr, D),
     epi_store(d_logits, V), 0);
  have_cache_ = caches;
  last_B_ = B;
  last_T_ = T;
  return RNET_OK;
}

// ------------------------------------------------------------------ backward
int Engine::head_backward(const float* d_dlogits, int N) {
  const int D = cfg_.d_model, V = cfg_.vocab_size;
  unsigned* err = rnet_status::device_error_word();
  cudaStream_t s = stream_;
  // src/resonance_net.cpp:428-442
  const bool bf = precision == 1;
  if (bf) PROF(PK_OTHER, 0, 6.0 * N * V, rnet_k::to_bf16(d_dlogits, dlogitsh_, (size_t)N * V, s));
  MM(N, D, V, kop(bf, d_dlogits, dlogitsh_, V), mop(bf, outw_, bf ? h16(outw_) : nullptr, D),
     epi_store(dnf_, D), 0);
  MM(V, D, N, mop(bf, d_dlogits, dlogitsh_, V), mop(bf, nf_, nfh_, D), epi_accum(g_outw_, D), 0);
  const float* XL = X_ + (size_t)cfg_.n_layers * N * D;
  PROF(PK_RMS_BWD, 0, 12.0 * N * D,
       rnet_k::rms_norm_bwd(dnf_, XL, fnorm_, rinvf_, dX_, g_fnorm_, N, D, 0, s, dXh_));
  return RNET_OK;
}

int Engine::layer_backward(int l, int B, int T) {
  const int N = B * T, D = cfg_.d_model, F = cfg_.d_ff, S = cfg_.n_slots, k = cfg_.slot_top_k;
  const LayerParams& w = W_[l];
  const LayerParams& g = G_[l];
  LayerAct& a = recompute_ ? act_[0] : act_[l];
  unsigned* err = rnet_status::device_error_word();
  cudaStream_t s = stream_;
  const float* Xl = X_ + (size_t)l * N * D;
  float* dKT = dKV_ + (size_t)l * 2 * S * D;
  float* dVT = dKT + (size_t)S * D;
  const double ND4 = 4.0 * N * D;
  const bool bf = precision == 1;
  auto W16 = [&](const float* p) { return bf ? h16(p) : nullptr; };
  // Weight-gradient GEMMs go to the side stream: fork() when their inputs are
  // ready on the main stream, join() before the main stream overwrites one
  // of those inputs (dX_ by the RMSNorm backward; dGU_ / dq_ / dPZH_ / dS_
  // only in later sublayers).
  auto fork = [&]() -> cudaError_t {
    if (prof_on_) return cudaSuccess;
    cudaError_t e = cudaEventRecord(ev_fork_, s);
    return e != cudaSuccess ? e : cudaStreamWaitEvent(wstream_, ev_fork_, 0);
  };
  auto join = [&]() -> cudaError_t {
    if (prof_on_) return cudaSuccess;
    cudaError_t e = cudaEventRecord(ev_join_, wstream_);
    return e != cudaSuccess ? e : cudaStreamWaitEvent(s, ev_join_, 0);
  };
  // 4. SwiGLU (src/resonance_net.cpp:468-490, src/swiglu_ffn.cu:88-152)
  // dH = dY W_down into the dG half of dGU, then the pointwise SwiGLU
  // gradient in place (a fused epilogue measured 4x slower: its cache reads
  // have too little memory-level parallelism in four epilogue warps)
  CK(fork());
  MM_W(D, F, N, mop(bf, dX_, dXh_, D), mop(bf, a.H, a.Hh, F), epi_accum(g.down, F));
  MM(N, F, D, kop(bf, dX_, dXh_, D), mop(bf, w.down, W16(w.down), F), epi_store(dGU_, 2 * F), 0);
  // bf16 mode: dG | dU written only as the bf16 copy the GEMMs read
  PROF(PK_OTHER, 0, (bf ? 16.0 : 20.0) * N * F,
       rnet_k::swiglu_bwd_pointwise(dGU_, 2 * F, a.G, a.U, N, F, s, bf ? dGUh_ : nullptr));
  CK(fork());
  MM_W(2 * F, D, N, mop(bf, dGU_, dGUh_, 2 * F), mop(bf, a.n4, a.n4h, D), epi_accum(g.gate, D));
  MM(N, D, 2 * F, kop(bf, dGU_, dGUh_, 2 * F), mop(bf, w.gate, W16(w.gate), D),
     epi_store(dsub_, D), 0);
  CK(join());
  PROF(PK_RMS_BWD, 0, 4 * ND4,
       rnet_k::rms_norm_bwd(dsub_, a.r3, w.n4, a.rinv4, dX_, g.n4, N, D, 1, s, dXh_));
  // 3. slot memory (:492-510, src/slot_memory.cu:171-244) — sparse top-k path
  CK(fork());
  MM_W(D, D, N, mop(bf, dX_, dXh_, D), mop(bf, a.r, a.rh, D), epi_accum(g.pout, D));
  MM(N, D, D, kop(bf, dX_, dXh_, D), mop(bf, w.pout, W16(w.pout), D), epi_store(dr_, D), 0);
  CK(cudaMemsetAsync(dKT, 0, 2 * (size_t)S * D * sizeof(float), s));  // dKT and dVT
  PROF(PK_SLOT_SPARSE_BWD, 8.0 * k * N * D, (2 + 4 * k) * ND4 + (bf ? 2.0 : 4.0) * N * D,
       rnet_k::slot_sparse_bwd(dr_, a.idx, a.w, VT_ + (size_t)l * S * D, KT_ + (size_t)l * S * D,
                               a.q, bf ? nullptr : dq_, dVT, dKT, N, D, S, k, err, s, dqh_));
  CK(fork());
  MM_W(D, D, N, mop(bf, dq_, dqh_, D), mop(bf, a.n3, a.n3h, D), epi_accum(g.pq, D));
  // dKT, dVT are adjacent [S, D] blocks of consecutive layers: both into
  // the gradient's keys / values in one launch
  PROF(PK_OTHER, 0, 32.0 * S * D,
       rnet_k::transpose_pairs(dKT, (size_t)S * D, 0, g.keys, g.vals, 0, 1, S, D, 1, s));
  MM(N, D, D, kop(bf, dq_, dqh_, D), mop(bf, w.pq, W16(w.pq), D), epi_store(dsub_, D), 0);
  CK(join());
  PROF(PK_RMS_BWD, 0, 4 * ND4,
       rnet_k::rms_norm_bwd(dsub_, a.r2, w.n3, a.rinv3, dX_, g.n3, N, D, 1, s, dXh_));
  // 2. MinGRU (:512-528, src/min_gru.cu:128-191)
  PROF(PK_SCAN_BWD, 0, 3 * ND4 + (bf ? 2.0 : 4.0) * 2 * N * D,
       rnet_k::gru_scan_bwd(dX_, a.z, a.h, nullptr, 0, nullptr, dPZH_, dPZH_ + D, 2 * D, g.bz,
                            g.bh, B, T, D, s, bf ? dPZHh_ : nullptr));
  CK(fork());
  MM_W(2 * D, D, N, mop(bf, dPZH_, dPZHh_, 2 * D), mop(bf, a.n2, a.n2h, D), epi_accum(g.Wz, D));
  MM(N, D, 2 * D, kop(bf, dPZH_, dPZHh_, 2 * D), mop(bf, w.Wz, W16(w.Wz), D),
     epi_store(dsub_, D), 0);
  CK(join());
  PROF(PK_RMS_BWD, 0, 4 * ND4,
       rnet_k::rms_norm_bwd(dsub_, a.r1, w.n2, a.rinv2, dX_, g.n2, N, D, 1, s, dXh_));
  // 1. causal conv (:530-545, src/causal_conv.cu:132-190)
  CK(fork());
  MM_W(D, D, N, mop(bf, dX_, dXh_, D),
       mop(bf, conv_quirk ? a.Sq : a.S, conv_quirk ? a.Sqh : a.Sh, D), epi_accum(g.mix, D));
  MM(N, D, D, kop(bf, dX_, dXh_, D), mop(bf, w.mix, W16(w.mix), D), epi_store(dS_, D), 0);
  PROF(PK_CONV_BWD, 100.0 * N * D, 3 * ND4,
       rnet_k::conv_bwd(dS_, a.n1, w.c3, w.c7, w.c15, dsub_, g.c3, g.c7, g.c15, conv_parts_, B, T,
                        D, 0, s));
  CK(join());
  PROF(PK_RMS_BWD, 0, 4 * ND4,
       rnet_k::rms_norm_bwd(dsub_, Xl, w.n1, a.rinv1, dX_, g.n1, N, D, 1, s, dXh_));
  return RNET_OK;
}

int Engine::backward(const float* d_dlogits, const int* d_tokens, int B, int T) {
  if (!have_cache_ || B != last_B_ || T != last_T_)
    return rnet_status::fail(RNET_ERR_ARG,
                             "backward: needs a preceding cached forward with the same B, T");
  const int N = B * T;
  int rc = head_backward(d_dlogits, N);
  if (rc) return rc;
  const size_t ND = (size_t)N * cfg_.d_model;
  // Gradient buckets: contiguous ranges of the flat gradient buffer, a layer
  // at a time from the last layer down, merged until a bucket holds at least
  // bucket_bytes_ (4 MB by default, RNET_DP_BUCKET_MB overrides), then
  // all-reduced on the comm stream while the backward goes on.
  if (bucket_bytes_ == 0) {
    const char* e = getenv("RNET_DP_BUCKET_MB");
    const double mb = e ? atof(e) : 4.0;
    bucket_bytes_ = (size_t)((mb > 0 ? mb : 4.0) * 1e6);
  }
  // bf16 mode: gradient buckets travel as bf16 (one staging buffer of the
  // largest bucket; the comm stream orders its reuse)
  __nv_bfloat16* c16 = nullptr;
  if (dist && precision == 1) {
    // a bucket stops growing once it reaches bucket_bytes_: at most that plus
    // one layer (or the head)
    const size_t need = bucket_bytes_ / sizeof(float) +
                        std::max(G_[0].count, 2 * (size_t)cfg_.vocab_size * cfg_.d_model +
                                                  (size_t)cfg_.d_model);
    if (comm16_count_ < need) {
      CK(cudaStreamSynchronize(stream_));
      cudaFree(comm16_);
      comm16_ = nullptr;
      CK(cudaMalloc(&comm16_, need * sizeof(__nv_bfloat16)));
      comm16_count_ = need;
    }
    c16 = comm16_;
  }
  size_t pend_lo = 0, pend_hi = 0;  // pending bucket [lo, hi) in floats
  auto flush = [&](bool force) -> int {
    if (!dist || pend_hi == pend_lo) return RNET_OK;
    if (!force && (pend_hi - pend_lo) * sizeof(float) < bucket_bytes_) return RNET_OK;
    const int r = dist_reduce_range(dist, grads_ + pend_lo, pend_hi - pend_lo, stream_, c16);
    pend_lo = pend_hi = 0;
    return r;
  };
  for (int l = cfg_.n_layers - 1; l >= 0; --l) {
    // recompute mode: the caches in act_[0] are the last layer's after the
    // forward; every other layer's are rebuilt from its kept input (the
    // recomputed output X[l+1] equals the stored one: same kernels, same
    // inputs, no atomics in the forward)
    if (recompute_ && l != cfg_.n_layers - 1) {
      rc = layer_forward(l, X_ + (size_t)l * ND, X_ + (size_t)(l + 1) * ND, act_[0], B, T, true);
      if (rc) return rc;
    }
    rc = layer_backward(l, B, T);
    if (rc) return rc;
    if (dist) {
      // layer l sits directly below the pending range (layer l + 1, ...)
      pend_hi = pend_hi == pend_lo ? G_[l].offset + G_[l].count : pend_hi;
      pend_lo = G_[l].offset;
      rc = flush(false);
      if (rc) return rc;
    }
  }
  PROF(PK_EMBED, 0, 4.0 * N * cfg_.d_model,
       rnet_k::embed_bwd(dX_, d_tokens, g_embed_, N, cfg_.vocab_size, cfg_.d_model, stream_));
  if (dist) {
    // the head (embedding, output, final norm) sits below layer 0
    if (pend_hi == pend_lo) pend_hi = G_[0].offset;
    pend_lo = 0;
    rc = flush(true);
    if (rc) return rc;
  }
  return RNET_OK;
}
int Engine::zero_grad() {
  CK(cudaMemsetAsync(grads_, 0, P_ * sizeof(float), stream_));
  return RNET_OK;
}

int Engine::step(float lr, float clip) {
  int world = 1;
  if (dist) {
    cudaEvent_t pa = nullptr;
    if (prof_on_) prof_begin(&pa);
    int rc = dist_wait(dist, stream_);
    if (rc) return rc;
    if (prof_on_) prof_end(pa, PK_COMM_WAIT, 0, 0);
    world = dist_world(dist);
  }
  const bool bf = precision == 1;
  if (warmup_ > 0) {
    const double f = (double)(step_count_ + 1) / warmup_;
    if (f < 1.0) lr = (float)(lr * f);
  }
  ++step_count_;
  PROF(PK_SGD, 2.0 * P_, (bf ? 18.0 : 16.0) * P_ + (velocity_ ? 8.0 * P_ : 0.0),
       rnet_k::sgd_clip_step(params_, grads_, P_, lr, clip, world, scratch_, norm_dev_, stream_,
                             bf ? params16_ : nullptr, velocity_, momentum_, weight_decay_));
  cudaEvent_t pa = nullptr;
  if (prof_on_) prof_begin(&pa);
  int rc = refresh_shadows_impl(bf);
  if (prof_on_) prof_end(pa, PK_OTHER, 0, 16.0 * 2 * cfg_.n_layers * cfg_.n_slots * cfg_.d_model);
  return rc;
}

int Engine::train_step(const int* d_in, const int* d_tgt, int B, int T, float lr, float clip,
                       float* d_loss_sum) {
  const int N = B * T;
  if (!train_graphs_ || dist || prof_on_ || (warmup_ > 0 && step_count_ < warmup_) || N <= 0 ||
      N > 64 * (cfg_.seq_len > 0 ? cfg_.seq_len : 256))
    return train_step_eager(d_in, d_tgt, B, T, lr, clip, d_loss_sum);
  int rc = ensure_capacity(N, true);  // may reallocate: never inside a capture
  if (rc) return rc;
  if (N > g_cap_) {
    if (train_exec_) cudaGraphExecDestroy(train_exec_);
    train_exec_ = nullptr;
    warm_valid_ = false;
    CK(cudaStreamSynchronize(stream_));
    cudaFree(g_in_);
    cudaFree(g_tgt_);
    g_in_ = g_tgt_ = nullptr;
    CK(cudaMalloc(&g_in_, N * sizeof(int)));
    CK(cudaMalloc(&g_tgt_, N * sizeof(int)));
    g_cap_ = N;
  }
  TrainKey key;
  key.B = B;
  key.T = T;
  key.lr = lr;
  key.clip = clip;
  key.arena = arena_;
  key.params16 = params16_;
  key.velocity = velocity_;
  key.momentum = momentum_;
  key.weight_decay = weight_decay_;
  key.precision = precision;
  key.recompute = recompute_;
  key.conv_quirk = conv_quirk;
  CK(cudaMemcpyAsync(g_in_, d_in, N * sizeof(int), cudaMemcpyDeviceToDevice, stream_));
  CK(cudaMemcpyAsync(g_tgt_, d_tgt, N * sizeof(int), cudaMemcpyDeviceToDevice, stream_));
  if (!(train_exec_ && key == train_key_)) {
    if (!(warm_valid_ && key == warm_key_)) {
      // first step with this key: eager (kernel attributes, tensor maps and
      // caches are set up outside any capture)
      warm_key_ = key;
      warm_valid_ = true;
      rc = train_step_eager(g_in_, g_tgt_, B, T, lr, clip, loss_dev_);
      if (rc) return rc;
      if (d_loss_sum)
        CK(cudaMemcpyAsync(d_loss_sum, loss_dev_, sizeof(float), cudaMemcpyDeviceToDevice,
                           stream_));
      return RNET_OK;
    }
    if (train_exec_) cudaGraphExecDestroy(train_exec_);
    train_exec_ = nullptr;
    const long long count0 = step_count_;
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    rc = train_step_eager(g_in_, g_tgt_, B, T, lr, clip, loss_dev_);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(stream_, &g);
    cudaGraphExec_t exec = nullptr;
    size_t nodes = 0;
    bool captured = rc == RNET_OK && ce == cudaSuccess && g &&
                    cudaGraphGetNodes(g, nullptr, &nodes) == cudaSuccess;
    size_t kernels = 0;  // launches counted: kernel nodes only (not the memset)
    if (captured && nodes) {
      std::vector<cudaGraphNode_t> list(nodes);
      captured = cudaGraphGetNodes(g, list.data(), &nodes) == cudaSuccess;
      for (size_t i = 0; captured && i < nodes; ++i) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(list[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
          ++kernels;
      }
    }
    captured = captured && cudaGraphInstantiate(&exec, g, 0) == cudaSuccess;
    if (g) cudaGraphDestroy(g);
    if (!captured) {
      // run eagerly from now on (the capture ran nothing)
      cudaGetLastError();
      train_graphs_ = false;
      step_count_ = count0;
      return train_step_eager(d_in, d_tgt, B, T, lr, clip, d_loss_sum);
    }
    train_exec_ = exec;
    train_nodes_ = kernels;
    train_key_ = key;
    // the capture advanced the host-side step count; the launch below is
    // that step
  } else {
    ++step_count_;
  }
  CK(cudaGraphLaunch(train_exec_, stream_));
  rnet_status::count_launch((unsigned)train_nodes_);
  if (d_loss_sum)
    CK(cudaMemcpyAsync(d_loss_sum, loss_dev_, sizeof(float), cudaMemcpyDeviceToDevice, stream_));
  return RNET_OK;
}

int Engine::train_step_eager(const int* d_in, const int* d_tgt, int B, int T, float lr, float clip,
                       float* d_loss_sum) {
  const int N = B * T, V = cfg_.vocab_size;
  if (N > 64 * (cfg_.seq_len > 0 ? cfg_.seq_len : 256))
    return rnet_status::fail(RNET_ERR_ARG, "train_step: batch*seq_len exceeds 64*seq_len");
  int rc = zero_grad();
  if (rc) return rc;
  rc = ensure_capacity(N, true);
  if (rc) return rc;
  rc = forward(d_in, logits_, B, T);
  if (rc) return rc;
  PROF(PK_CE, 0, 8.0 * N * V,
       rnet_k::cross_entropy(logits_, d_tgt, d_loss_sum ? d_loss_sum : loss_dev_, dlogits_,
                             1.0f / (float)N, conv_parts_, N, V, rnet_status::device_error_word(),
                             stream_));
  rc = backward(dlogits_, d_in, B, T);
  if (rc) return rc;
  return step(lr, clip);
}

// ------------------------------------------------------------------ decode
int Engine::decoder_init(Decoder* d, int M) {
  if (M <= 0) return rnet_status::fail(RNET_ERR_ARG, "decoder: n_streams must be > 0");
  const size_t D = cfg_.d_model, F = cfg_.d_ff, V = cfg_.vocab_size, L = cfg_.n_layers;
  const size_t k = cfg_.slot_top_k, m = M;
  if (k != 2) return rnet_status::fail(RNET_ERR_UNSUPPORTED, "decoder: slot_top_k must be 2");
  if (cfg_.n_slots % 4 || D % 4)
    return rnet_status::fail(RNET_ERR_UNSUPPORTED, "decoder: n_slots and d_model must be % 4");
  d->M = M;
  d->floats_per_layer = m * 15 * D;
  std::vector<std::pair<void**, size_t>> plan;
  auto f = [&](float** p, size_t n) { plan.push_back({(void**)p, n * sizeof(float)}); };
  f(&d->state, L * d->floats_per_layer);
  f(&d->x, m * D); f(&d->n, m * D); f(&d->S, m * D); f(&d->P, 2 * m * D); f(&d->q, m * D);
  f(&d->r, m * D); f(&d->G, m * F); f(&d->U, m * F); f(&d->H, m * F); f(&d->logits, m * V);
  f(&d->GU, m * 2 * F); f(&d->scores, m * (size_t)cfg_.n_slots);
  f(&d->w, m * k);
  f(&d->KqT, L * cfg_.n_slots * D);
  f(&d->VP, L * cfg_.n_slots * D);
  plan.push_back({(void**)&d->idx, m * k * sizeof(int)});
  plan.push_back({(void**)&d->tok, m * sizeof(int)});
  plan.push_back({(void**)&d->pos, sizeof(int)});
  size_t total = 0;
  for (auto& e : plan) total += (e.second + 255) & ~size_t(255);
  CK(cudaMalloc(&d->arena, total));
  CK(cudaMemsetAsync(d->arena, 0, total, stream_));
  // split-K workspace of the decode step's short-M GEMMs (the step is
  // captured into a graph, which cannot allocate). splits <= SMs / tiles and a
  // tile covers 128 x 128 outputs, so splits * M * N <= SMs * 128 * 128.
  CK(rnet_gemm::reserve_workspace(stream_, (size_t)rnet_gemm::num_sms() * 128 * 128));
  char* p = (char*)d->arena;
  for (auto& e : plan) {
    *e.first = p;
    p += (e.second + 255) & ~size_t(255);
  }
  return RNET_OK;
}

void Engine::decoder_free(Decoder* d) {
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  cudaStreamSynchronize(stream_);
  cudaFree(d->arena);
  d->arena = nullptr;
  d->exec = nullptr;
  d->graph = nullptr;
}

int Engine::prefill(Decoder* d, const int* d_tokens, int T) {
  if (T <= 0) return rnet_status::fail(RNET_ERR_ARG, "prefill: empty prompt");
  const int M = d->M, N = M * T, D = cfg_.d_model, V = cfg_.vocab_size;
  int rc = ensure_capacity(N, false);
  if (rc) return rc;
  cudaStream_t s = stream_;
  unsigned* err = rnet_status::device_error_word();
  const size_t ND = (size_t)N * D;
  PROF(PK_EMBED, 0, 4.0 * ND, rnet_k::embed_fwd(d_tokens, embed_, X_, N, V, D, err, s));
  for (int l = 0; l < cfg_.n_layers; ++l) {
    const float* Xl = X_ + (size_t)(l & 1) * ND;
    float* Xn = X_ + (size_t)((l + 1) & 1) * ND;
    rc = layer_forward(l, Xl, Xn, act_[0], M, T, false);
    if (rc) return rc;
    float* st = d->state + (size_t)l * d->floats_per_layer;
    CK(rnet_k::decode_extract_state(act_[0].n1, act_[0].h, st, st + (size_t)M * 14 * D, M, T, D,
                                    s));
  }
  have_cache_ = false;
  // fold the slot path's fixed projections for the decode steps:
  // KqT[s, e] = sum_d KT[s, d] proj_q[d, e], VP[s, j] = sum_d VT[s, d] proj_out[j, d]
  const int S = cfg_.n_slots;
  for (int l = 0; l < cfg_.n_layers; ++l) {
    const size_t o = (size_t)l * S * D;
    CK(rnet_k::fold_rows(KT_ + o, W_[l].pq, (size_t)D, 1, d->KqT + o, S, D, D, s));
    CK(rnet_k::fold_rows(VT_ + o, W_[l].pout, 1, (size_t)D, d->VP + o, S, D, D, s));
  }
  const float* XL = X_ + (size_t)(cfg_.n_layers & 1) * ND;
  CK(rnet_k::last_rows(XL, d->x, M, T, D, s));
  CK(rnet_k::rms_norm_fwd(d->x, fnorm_, d->n, nullptr, M, D, cfg_.rms_eps, s));
  MM(M, V, D, kmaj(d->n, D), kmaj(outw_, D), epi_store(d->logits, V), 0);
  CK(cudaMemcpyAsync(d->pos, &T, sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));  // &T is a stack value
  CK(rnet_k::sample_rows(d->logits, M, V, d->temperature, d->top_p, d->seed, d->tok, d->pos, 0,
                         s));
  return RNET_OK;
}

int Engine::decode_step(Decoder* d, const int* d_tokens) {
  const int M = d->M, D = cfg_.d_model, F = cfg_.d_ff, S = cfg_.n_slots, V = cfg_.vocab_size;
  const int L = cfg_.n_layers;
  const float eps = cfg_.rms_eps;
  cudaStream_t s = stream_;
  unsigned* err = rnet_status::device_error_word();
  if (d_tokens) CK(cudaMemcpyAsync(d->tok, d_tokens, M * sizeof(int), cudaMemcpyDeviceToDevice, s));
  CK(rnet_k::embed_fwd(d->tok, embed_, d->x, M, V, D, err, s));
  CK(rnet_k::rms_norm_fwd(d->x, W_[0].n1, d->n, nullptr, M, D, eps, s));
  // Every residual update also writes the next sublayer's RMSNorm of x into
  // d->n (in the kernel that sums the split-K partials), so no norm has a
  // launch of its own after the first.
  auto with_norm = [&](Epilogue e, const float* nw) {
    e.nw = nw;
    e.ny = d->n;
    e.eps = eps;
    return e;
  };
  for (int l = 0; l < L; ++l) {
    const LayerParams& w = W_[l];
    float* ring = d->state + (size_t)l * d->floats_per_layer;
    float* h = ring + (size_t)M * 14 * D;
    const size_t so = (size_t)l * S * D;
    // layer 0's conv step here; later layers' ran where the previous layer's
    // down projection was summed (below)
    if (l == 0) CK(rnet_k::decode_conv(d->n, ring, d->pos, w.c3, w.c7, w.c15, d->S, M, D, s));
    MMS(M, D, D, kmaj(d->S, D), kmaj(w.mix, D), with_norm(epi_accum(d->x, D), w.n2), 0, 1);
    {
      // gate pre-activations -> GRU state update + residual (+ norm 3) where
      // the split-K partials are summed
      Epilogue e;
      e.kind = EPI_PAIR_GRU;
      e.C = d->P;
      e.ldf = D;
      e.b0 = w.bz;
      e.b1 = w.bh;
      e.state = h;
      e.xres = d->x;
      MM(M, 2 * D, D, kmaj(d->n, D), kmaj(w.Wz, D), with_norm(e, w.n3), 0);
    }
    {
      // scores = n . (K proj_q)^T: the partial planes go straight to the
      // top-2 kernel, which also gathers the folded values into x (+ norm 4)
      int planes = 1;
      const float* pl = nullptr;
      Epilogue e = epi_store(d->scores, S);
      e.splits_out = &planes;
      e.planes_out = &pl;
      MM(M, S, D, kmaj(d->n, D), kmaj(d->KqT + so, D), e, 0);
      CK(rnet_k::topk2_gather_residual_norm(pl, planes, d->idx, d->w, M, S, d->VP + so, d->x, D,
                                            w.n4, d->n, eps, s));
    }
    // gate|up as one [2F, D] operand (adjacent in the parameter buffer)
    {
      Epilogue e;  // gate|up -> silu(gate) * up where the partials are summed
      e.kind = EPI_PAIR_SILU;
      e.C = d->GU;
      e.H = d->H;
      e.ldf = F;
      MM(M, 2 * F, D, kmaj(d->n, D), kmaj(w.gate, D), e, 0);
    }
    if (l + 1 < L) {
      // x += H down^T, n = RMSNorm_1(x) of the next layer, and that layer's
      // conv step on n, all where the split-K partials are summed
      const LayerParams& wn = W_[l + 1];
      Epilogue e = with_norm(epi_accum(d->x, D), wn.n1);
      e.cw3 = wn.c3;
      e.cw7 = wn.c7;
      e.cw15 = wn.c15;
      e.ring = d->state + (size_t)(l + 1) * d->floats_per_layer;
      e.pos = d->pos;
      e.conv_out = d->S;
      MMS(M, D, F, kmaj(d->H, F), kmaj(w.down, F), e, 0, 1);
    } else {
      MMS(M, D, F, kmaj(d->H, F), kmaj(w.down, F), with_norm(epi_accum(d->x, D), fnorm_), 0, 1);
    }
  }
  MM(M, V, D, kmaj(d->n, D), kmaj(outw_, D), epi_store(d->logits, V), 0);
  CK(rnet_k::sample_rows(d->logits, M, V, d->temperature, d->top_p, d->seed, d->tok, d->pos, 1,
                         s));
  return RNET_OK;
}

int Engine::generate(Decoder* d, int n_steps, int* d_out, bool use_graph) {
  cudaStream_t s = stream_;
  if (use_graph && !d->exec) {
    // one eager step first so every kernel attribute / tensor map is set up,
    // then capture the step (all arguments are fixed device pointers; the
    // position lives in device memory and is advanced by the argmax kernel)
    int rc = decode_step(d, nullptr);
    if (rc) return rc;
    if (d_out) CK(cudaMemcpyAsync(d_out, d->tok, d->M * sizeof(int), cudaMemcpyDeviceToDevice, s));
    --n_steps;
    d_out = d_out ? d_out + d->M : nullptr;
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    rc = decode_step(d, nullptr);
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamEndCapture(s, &g);
    if (rc) return rc;
    CK(ce);
    d->graph = g;
    size_t nodes = 0;
    CK(cudaGraphGetNodes(g, nullptr, &nodes));
    d->graph_kernels = (int)nodes;  // the captured step contains kernel nodes only
    CK(cudaGraphInstantiate(&d->exec, g, 0));
  }
  for (int i = 0; i < n_steps; ++i) {
    if (d->exec) {
      CK(cudaGraphLaunch(d->exec, s));
      rnet_status::count_launch((unsigned)d->graph_kernels);
    } else {
      int rc = decode_step(d, nullptr);
      if (rc) return rc;
    }
    if (d_out)
      CK(cudaMemcpyAsync(d_out + (size_t)i * d->M, d->tok, d->M * sizeof(int),
                         cudaMemcpyDeviceToDevice, s));
  }
  return RNET_OK;
}

int Engine::set_optimizer(float momentum, float weight_decay, int warmup_steps) {
  if (!(momentum >= 0.0f && momentum < 1.0f) || !(weight_decay >= 0.0f) || warmup_steps < 0)
    return rnet_status::fail(RNET_ERR_ARG,
                             "set_optimizer: need 0 <= momentum < 1, weight_decay >= 0, "
                             "warmup_steps >= 0");
  momentum_ = momentum;
  weight_decay_ = weight_decay;
  warmup_ = warmup_steps;
  step_count_ = 0;
  CK(cudaStreamSynchronize(stream_));
  if (momentum > 0.0f) {
    if (!velocity_) CK(cudaMalloc(&velocity_, P_ * sizeof(float)));
    CK(cudaMemsetAsync(velocity_, 0, P_ * sizeof(float), stream_));
  } else {
    cudaFree(velocity_);
    velocity_ = nullptr;
  }
  return RNET_OK;
}

int Engine::set_recompute(bool on) {
  recompute_ = on;
  have_cache_ = false;
  return RNET_OK;
}

int Engine::topk(int layer, int** idx, float** w) {
  if (!have_cache_ || layer < 0 || layer >= cfg_.n_layers)
    return rnet_status::fail(RNET_ERR_ARG, "topk: no cached forward or bad layer");
  if (recompute_)
    return rnet_status::fail(RNET_ERR_ARG, "topk: selections are not kept with recompute on");
  *idx = act_[layer].idx;
  *w = act_[layer].w;
  return RNET_OK;
}

// ------------------------------------------------------------------ checkpoint
// Byte layout of the reference (src/resonance_net.cpp:743-782): the 40-byte
// ModelConfig, then every tensor in order as raw fp32 — here one contiguous
// write because the parameters already live in that order.
int Engine::save(const char* path) {
  std::vector<float> h(P_);
  CK(cudaMemcpyAsync(h.data(), params_, P_ * sizeof(float), cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  FILE* f = fopen(path, "wb");
  if (!f) return rnet_status::fail(RNET_ERR_IO, std::string("cannot open for write: ") + path);
  bool ok = fwrite(&cfg_, sizeof(cfg_), 1, f) == 1;
  ok = ok && fwrite(h.data(), sizeof(float), P_, f) == P_;
  ok = (fclose(f) == 0) && ok;
  if (!ok) return rnet_status::fail(RNET_ERR_IO, std::string("short write: ") + path);
  return RNET_OK;
}

int Engine::save_async(const char* path) {
  int rc = save_wait();
  if (rc) return rc;
  if (!snap_) {
    CK(cudaMalloc(&snap_, P_ * sizeof(float)));
    CK(cudaMallocHost(&snap_host_, P_ * sizeof(float)));
    CK(cudaStreamCreateWithFlags(&save_stream_, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&snap_ready_, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&host_ready_, cudaEventDisableTiming));
  }
  // the snapshot is ordered on the model stream: the next SGD update cannot
  // overtake it
  CK(cudaMemcpyAsync(snap_, params_, P_ * sizeof(float), cudaMemcpyDeviceToDevice, stream_));
  CK(cudaEventRecord(snap_ready_, stream_));
  CK(cudaStreamWaitEvent(save_stream_, snap_ready_, 0));
  CK(cudaMemcpyAsync(snap_host_, snap_, P_ * sizeof(float), cudaMemcpyDeviceToHost,
                     save_stream_));
  CK(cudaEventRecord(host_ready_, save_stream_));
  const std::string file(path);
  const rnet_model_config cfg = cfg_;
  save_status_ = RNET_OK;
  save_msg_.clear();
  save_thread_ = new std::thread([this, file, cfg]() {
    if (cudaEventSynchronize(host_ready_) != cudaSuccess) {
      save_status_ = RNET_ERR_CUDA;
      save_msg_ = "save_async: snapshot copy failed";
      return;
    }
    FILE* f = fopen(file.c_str(), "wb");
    if (!f) {
      save_status_ = RNET_ERR_IO;
      save_msg_ = "cannot open for write: " + file;
      return;
    }
    bool ok = fwrite(&cfg, sizeof(cfg), 1, f) == 1;
    ok = ok && fwrite(snap_host_, sizeof(float), P_, f) == P_;
    ok = (fclose(f) == 0) && ok;
    if (!ok) {
      save_status_ = RNET_ERR_IO;
      save_msg_ = "short write: " + file;
    }
  });
  return RNET_OK;
}

int Engine::save_wait() {
  if (!save_thread_) return RNET_OK;
  std::thread* t = static_cast<std::thread*>(save_thread_);
  t->join();
  delete t;
  save_thread_ = nullptr;
  if (save_status_) return rnet_status::fail(save_status_, save_msg_);
  return RNET_OK;
}

int Engine::load_weights(const char* path) {
  FILE* f = fopen(path, "rb");
  if (!f) return rnet_status::fail(RNET_ERR_IO, std::string("cannot open: ") + path);
  rnet_model_config c;
  if (fread(&c, sizeof(c), 1, f) != 1) {
    fclose(f);
    return rnet_status::fail(RNET_ERR_IO, "checkpoint: truncated header");
  }
  if (c.d_model != cfg_.d_model || c.n_layers != cfg_.n_layers || c.d_ff != cfg_.d_ff ||
      c.n_slots != cfg_.n_slots || c.vocab_size != cfg_.vocab_size) {
    fclose(f);
    return rnet_status::fail(RNET_ERR_IO, "checkpoint: config does not match this model");
  }
  std::vector<float> h(P_);
  const size_t got = fread(h.data(), sizeof(float), P_, f);
  const bool extra = fgetc(f) != EOF;
  fclose(f);
  if (got != P_) return rnet_status::fail(RNET_ERR_IO, "checkpoint: truncated tensor data");
  if (extra) return rnet_status::fail(RNET_ERR_IO, "checkpoint: trailing bytes after tensors");
  return set_params_host(h.data(), P_);
}

}  // namespace rnet_engine
