// ResonanceNet model engine: parameters, gradients, activation caches and the
// per-layer forward / backward / SGD schedule on one CUDA stream.
//
// Parameters and gradients each live in ONE flat device buffer laid out in
// checkpoint tensor order (reference src/resonance_net.cpp:759-778), so a
// checkpoint is one read/write, the optimizer is one pass, and data-parallel
// gradient buckets are contiguous ranges. Within a layer Wz|Wh and gate|up
// are adjacent in that order, which the fused GEMMs use as [2D,D] / [2F,D].
#pragma once
#include <cuda_bf16.h>
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
  // bf16 copies of the GEMM operands (bf16 mode only, else null)
  __nv_bfloat16 *n2h, *n3h, *n4h, *Sh, *Sqh, *qh, *rh, *Hh;
};

class DistComm;  // dist.cu

// Per-kernel-class event timing (enabled on demand; one event pair per launch
// group, on the engine stream).
enum ProfKind {
  PK_GEMM = 0,
  PK_SCAN_FWD,
  PK_SCAN_BWD,
  PK_CONV_FWD,
  PK_CONV_BWD,
  PK_RMS_FWD,
  PK_RMS_BWD,
  PK_SLOT_GATHER,
  PK_SLOT_SPARSE_BWD,
  PK_EMBED,
  PK_CE,
  PK_SGD,
  PK_OTHER,
  PK_COMM_WAIT,  // data parallel: compute stream stalled on the last all-reduce
  PK_COUNT
};

struct ProfStats {
  double ms[PK_COUNT];
  double flops[PK_COUNT];
  double bytes[PK_COUNT];
  long long launches[PK_COUNT];
};

// Recurrent decode state and buffers for M lock-step streams.
struct Decoder {
  int M = 0;
  float* state = nullptr;  // per layer: ring [M][14][D] then h [M][D]
  size_t floats_per_layer = 0;
  float *x, *n, *S, *P, *q, *r, *G, *U, *H, *logits;
  float *GU, *scores;  // [M, 2F] gate|up pre-activations, [M, S] slot scores
  // per layer [S, D]: keys folded with proj_q (scores = n . KqT[s]) and
  // values folded with proj_out (slot output = sum_j w_j VP[i_j]), made at
  // prefill from the weights of that moment
  float *KqT, *VP;
  int* idx;
  float* w;
  int* tok;  // current / next token per stream
  int* pos;  // device scalar: index of the token being processed
  void* arena = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraph_t graph = nullptr;
  int graph_kernels = 0;
  // next-token rule: greedy when temperature <= 0, else temperature + top-p
  // sampling (src/main.cpp:327-360) with a counter-based uniform per
  // (seed, stream, position)
  float temperature = 0.0f;
  float top_p = 1.0f;
  unsigned long long seed = 0;
};

class Engine {
 public:
  // ---- decode (O(1) recurrent state) ----
  int decoder_init(Decoder* d, int M);
  void decoder_free(Decoder* d);
  // Chunked-scan forward over d_tokens [M, T]; leaves the state after T
  // tokens, last-position logits in d->logits and their argmax in d->tok.
  int prefill(Decoder* d, const int* d_tokens, int T);
  // One token per stream (d_tokens, or the previous argmax when null);
  // logits in d->logits, argmax in d->tok.
  int decode_step(Decoder* d, const int* d_tokens);
  // n_steps greedy steps; d_out [n_steps][M] receives the generated tokens.
  int generate(Decoder* d, int n_steps, int* d_out, bool use_graph);

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
  // Single-GPU steps run from a captured CUDA graph once the same (B, T, lr,
  // clip, configuration) repeats: the inputs are copied into engine buffers
  // first and the loss sum out afterwards, so the graph holds no caller
  // pointer. Data-parallel, profiled and warmup steps run eagerly, and so
  // does everything with RNET_TRAIN_GRAPH=0.
  int train_step(const int* d_in, const int* d_tgt, int B, int T, float lr, float clip,
                 float* d_loss_sum);
  // the step's launches in order (what the graph captures)
  int train_step_eager(const int* d_in, const int* d_tgt, int B, int T, float lr, float clip,
                       float* d_loss_sum);

  // Optimizer extensions (off by default: the reference's plain SGD with
  // clipping, src/resonance_net.cpp:551-663): momentum, weight decay added
  // after clipping, and a linear learning-rate warmup over warmup_steps
  // (lr * min(1, (t + 1) / warmup) at step t; the reference parses
  // TrainConfig::warmup_steps but never applies it). Resets the step count
  // and the velocity.
  int set_optimizer(float momentum, float weight_decay, int warmup_steps);
  int save(const char* path);
  // Checkpoint without stalling training: the parameters are snapshotted on
  // the model stream (device copy, ordered after everything queued so far),
  // then copied to pinned host memory on a side stream and written by a host
  // thread. save_wait() joins it and returns its status. One save in flight.
  int save_async(const char* path);
  int save_wait();
  int load_weights(const char* path);  // config in file must match

  int topk(int layer, int** idx, float** w);
  cudaStream_t stream() const { return stream_; }
  const rnet_model_config& config() const { return cfg_; }

  bool conv_quirk = true;  // reference dmix operand (S + c7 + c15)
  // GEMM arithmetic: 0 = fp32-accurate (3xTF32, default); 1 = bf16: every
  // GEMM operand of the train step is a bf16 copy in memory (weights: a bf16
  // shadow of the fp32 master parameters, refreshed by the SGD update;
  // activations: bf16 side outputs of their producers), read by TMA as bf16
  // tiles into kind::f16 MMAs with fp32 accumulation. Everything else
  // (norms, scan, conv, slot top-2 / gather, loss, optimizer) stays fp32.
  int precision = 0;
  int set_precision(int p);
  DistComm* dist = nullptr;

  // workspace capacity in tokens
  int ensure_capacity(int N, bool with_caches);

  // Activation recompute: keep only the layer inputs X[0..L] from the
  // forward and recompute each layer's caches right before its backward
  // (one layer of caches in memory instead of L; one extra forward per step).
  int set_recompute(bool on);
  bool recompute() const { return recompute_; }

  // profiling
  void profile_enable(bool on) { prof_on_ = on; }
  int profile_read(ProfStats* out, bool reset);

 private:
  struct ProfRec {
    int kind;
    double flops, bytes;
    cudaEvent_t a, b;
  };
  bool prof_on_ = false;
  std::vector<ProfRec> prof_;
  std::vector<cudaEvent_t> ev_pool_;
  size_t ev_used_ = 0;
  cudaEvent_t prof_event();
  void prof_begin(cudaEvent_t* a);
  void prof_end(cudaEvent_t a, int kind, double flops, double bytes);

  int gemm_err(cudaError_t e, const char* what);
  // train: keep the activation caches the backward reads (scan keeps e = h~ -
  // h_prev in LayerAct::h); otherwise LayerAct::h holds h (prefill)
  int layer_forward(int l, const float* Xl, float* Xn, LayerAct& a, int B, int T, bool train);
  int layer_backward(int l, int B, int T);
  int head_backward(const float* d_dlogits, int N);

  rnet_model_config cfg_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaStream_t wstream_ = nullptr;  // backward weight-gradient GEMMs
  cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
  size_t P_ = 0;
  float* params_ = nullptr;
  float* grads_ = nullptr;
  float *embed_, *outw_, *fnorm_, *g_embed_, *g_outw_, *g_fnorm_;
  std::vector<LayerParams> W_, G_;
  float* KT_ = nullptr;  // [L][S][D]
  __nv_bfloat16* params16_ = nullptr;  // bf16 shadow of params_ (bf16 mode)
  __nv_bfloat16* KT16_ = nullptr;      // bf16 shadow of KT_ (bf16 mode)
  __nv_bfloat16* h16(const float* p) const { return params16_ + (p - params_); }
  int refresh_shadows_impl(bool params16_current);
  float* VT_ = nullptr;
  float* dKV_ = nullptr;  // [L][keys | values][S][D] scatter gradients
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
  __nv_bfloat16 *nfh_ = nullptr, *dlogitsh_ = nullptr, *dXh_ = nullptr, *dGUh_ = nullptr,
                *dqh_ = nullptr, *dPZHh_ = nullptr;
  bool cap_bf16_ = false;
  bool recompute_ = false;
  float momentum_ = 0.0f, weight_decay_ = 0.0f;
  int warmup_ = 0;
  long long step_count_ = 0;
  // captured train step (see train_step)
  struct TrainKey {
    int B = 0, T = 0;
    float lr = 0.f, clip = 0.f;
    const void* arena = nullptr;
    const void* params16 = nullptr;
    const void* velocity = nullptr;
    float momentum = 0.f, weight_decay = 0.f;
    int precision = 0;
    bool recompute = false, conv_quirk = false;
    bool operator==(const TrainKey& o) const {
      return B == o.B && T == o.T && lr == o.lr && clip == o.clip && arena == o.arena &&
             params16 == o.params16 && velocity == o.velocity && momentum == o.momentum &&
             weight_decay == o.weight_decay && precision == o.precision &&
             recompute == o.recompute && conv_quirk == o.conv_quirk;
    }
  };
  bool train_graphs_ = true;
  cudaGraphExec_t train_exec_ = nullptr;
  size_t train_nodes_ = 0;
  TrainKey train_key_, warm_key_;
  bool warm_valid_ = false;
  int* g_in_ = nullptr;  // the graph's token inputs / targets
  int* g_tgt_ = nullptr;
  int g_cap_ = 0;
  float* velocity_ = nullptr;
  // asynchronous save
  float* snap_ = nullptr;   // device snapshot of params_
  float* snap_host_ = nullptr;  // pinned
  cudaStream_t save_stream_ = nullptr;
  cudaEvent_t snap_ready_ = nullptr, host_ready_ = nullptr;
  void* save_thread_ = nullptr;  // std::thread*
  int save_status_ = 0;
  std::string save_msg_;
  size_t bucket_bytes_ = 0;  // data-parallel bucket size (0: read RNET_DP_BUCKET_MB, default 4)
  __nv_bfloat16* comm16_ = nullptr;  // bf16 all-reduce staging (bf16 mode, DP)
  size_t comm16_count_ = 0;
  bool cap_recompute_ = false;
  bool have_cache_ = false;
  int last_B_ = 0, last_T_ = 0;
};

}  // namespace rnet_engine
