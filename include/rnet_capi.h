/*
 * rnet_capi.h — the C ABI of the B200 (sm_100a) ResonanceNet library
 * (librnet_b200.so). Plain pointers and sizes only; every entry point returns
 * RNET_OK (0) or a negative status and records a message for rnet_last_error().
 *
 * Pointers named d_* / documented as "device" are CUDA device pointers on the
 * current device; `stream` is a cudaStream_t passed as void* (NULL = legacy
 * default stream). Work is asynchronous on that stream unless stated.
 *
 * The C++ drop-in headers (layers.h, resonance_net.h, dist.h) are implemented
 * on top of these functions; a ctypes/cffi binding needs only this file.
 */
#ifndef RNET_CAPI_H
#define RNET_CAPI_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RNET_OK 0
#define RNET_ERR_ARG -1         /* invalid argument / unsupported shape */
#define RNET_ERR_CUDA -2        /* CUDA runtime error (message has details) */
#define RNET_ERR_NCCL -3        /* NCCL error or NCCL library not loadable */
#define RNET_ERR_TIMEOUT -4     /* host-side rendezvous / collective deadline */
#define RNET_ERR_IO -5          /* checkpoint file error, short or malformed file */
#define RNET_ERR_DEVICE -6      /* a kernel raised the device error word */
#define RNET_ERR_UNSUPPORTED -7 /* configuration not implemented */

/* ------------------------------------------------------------------ status */

/* Message of the most recent failing call on this thread ("" if none). */
const char* rnet_last_error(void);

/* Library ABI version (major*100 + minor). */
int rnet_abi_version(void);

/* Number of CUDA kernels this library has launched in this process. */
int rnet_kernel_launches(unsigned long long* n);

/* Read (and optionally clear) the device error word of the current device:
 * bit 0 = a bounded wait timed out, bit 1 = out-of-range index seen,
 * bit 2 = TMEM allocation failed. Synchronises the device. */
int rnet_device_error(unsigned* word, int clear);

/* Self-test of the bounded-wait failure path (no reference counterpart): runs
 * n_ctas CTAs shaped like the pipelined kernels (a TMEM-owning warp and
 * waiters on an mbarrier) and waits on a barrier that nothing arrives on
 * (arrive = 0) or that one thread arrives on (arrive = 1), with a wait limit
 * of timeout_us. A run-out wait sets bit 0 of the device error word, the CTA
 * frees its TMEM and returns; *timed_out_ctas receives how many CTAs gave up.
 * Synchronises the device. */
int rnet_selftest_bounded_wait(int arrive, unsigned timeout_us, int n_ctas,
                               unsigned* timed_out_ctas);

/* ------------------------------------------------------------------ GEMM engine
 * C[M,N] (op)= alpha * A[M,K] * B[N,K]^T on the tcgen05 3xTF32 engine.
 * a_mn_major = 0: A(i,k) = A[i*lda + k]; 1: A(i,k) = A[k*lda + i]  (same for B).
 * op: 0 = store, 1 = accumulate (C += ...), 2 = residual (C = R + ...).
 * lda/ldb must be multiples of 4 and A/B 16-byte aligned. */
int rnet_gemm_f32(int M, int N, int K, const float* A, int lda, int a_mn_major, const float* B,
                  int ldb, int b_mn_major, float* C, int ldc, const float* R, int ldr, int op,
                  float alpha, void* stream);

/* C[M,N] (op)= alpha * A[M,K] * B[N,K]^T with bf16 A and B (same majors as
 * rnet_gemm_f32; row pitch a multiple of 8 elements, 16-byte aligned) on the
 * tcgen05 kind::f16 path: bf16 tiles staged by TMA straight from memory, fp32
 * accumulation, fp32 C. C16 (optional, op 0 / 2): also store the result as
 * bf16 with row pitch ldc. No counterpart in the reference (fp32 only). */
int rnet_gemm_bf16(int M, int N, int K, const void* A, int lda, int a_mn_major, const void* B,
                   int ldb, int b_mn_major, float* C, int ldc, const float* R, int ldr, int op,
                   float alpha, void* C16, void* stream);

/* Tile shape selection of the GEMM engine for every later call in this
 * process: 0 = automatic (CTA pairs, one 256-row MMA over two SMs, whenever
 * M > 128; single-CTA 128-row tiles otherwise), 1 = always single-CTA,
 * 2 = always CTA pairs. Results are identical up to fp32 summation order.
 * No counterpart in the reference (its GEMMs are cuBLAS calls). */
int rnet_gemm_set_cta_group(int cta_group);

/* Arithmetic of later rnet_gemm_f32 calls in this process: 0 = fp32-accurate
 * (default), 1 = bf16 operands with fp32 accumulation. */
int rnet_gemm_set_precision(int precision);

/* ------------------------------------------------------------------ layer ops
 * One entry per function of the reference's include/layers.h:28-153, same
 * argument meaning, same accumulate/overwrite contract:
 *   overwrite: every *_forward output and cache, rms_norm_backward dx,
 *              cross_entropy loss (sum over tokens) and dlogits;
 *   accumulate (+=): every parameter gradient, and dx of causal_conv /
 *              min_gru / slot_memory / swiglu backward.
 * All pointers are device pointers; temporaries are stream-ordered. The
 * cuBLAS handle of the reference signatures has no counterpart here. */
int rnet_rms_norm_forward(const float* x, const float* w, float* y, float* rms_cache,
                          int batch_seq, int dim, float eps, void* stream);
int rnet_rms_norm_backward(const float* dy, const float* x, const float* w,
                           const float* rms_cache, float* dx, float* dw, int batch_seq, int dim,
                           void* stream);
int rnet_embed_forward(const int* tokens, const float* table, float* output, int batch_seq,
                       int vocab, int dim, void* stream);
int rnet_embed_backward(const float* dout, const int* tokens, float* dtable, int batch_seq,
                        int vocab, int dim, void* stream);
/* output[M,N] = input[M,K] * weight[N,K]^T */
int rnet_linear_forward(const float* input, const float* weight, float* output, int M, int N,
                        int K, void* stream);
/* conv_buf [3, B*T, D] receives {S = c3+c7+c15, c7, c15} like the reference. */
int rnet_causal_conv_forward(const float* x, float* y, const float* conv3_w,
                             const float* conv7_w, const float* conv15_w, const float* mix_w,
                             float* conv_buf, int batch, int seq_len, int dim, void* stream);
/* dmix_quirk = 1 reproduces the reference's mix-weight gradient, which uses
 * S + c7 + c15 (src/causal_conv.cu:155-168); 0 uses S (the exact gradient). */
int rnet_causal_conv_backward(const float* dy, const float* x, const float* conv3_w,
                              const float* conv7_w, const float* conv15_w, const float* mix_w,
                              const float* conv_buf, float* dx, float* d_conv3_w,
                              float* d_conv7_w, float* d_conv15_w, float* d_mix_w, int batch,
                              int seq_len, int dim, int dmix_quirk, void* stream);
int rnet_min_gru_forward(const float* x, float* y, const float* Wz, const float* Wh,
                         const float* bz, const float* bh, float* z_cache, float* h_cache,
                         int batch, int seq_len, int dim, void* stream);
int rnet_min_gru_backward(const float* dy, const float* x, const float* Wz, const float* Wh,
                          const float* bz, const float* bh, const float* z_cache,
                          const float* h_cache, float* dx, float* dWz, float* dWh, float* dbz,
                          float* dbh, int batch, int seq_len, int dim, void* stream);
/* scores_cache may be NULL (scores are then not materialised; top_k == 2). */
int rnet_slot_memory_forward(const float* x, float* y, const float* slot_keys,
                             const float* slot_values, const float* proj_q,
                             const float* proj_out, float* q_cache, float* scores_cache,
                             int* topk_idx_cache, float* topk_w_cache, int batch, int seq_len,
                             int dim, int n_slots, int top_k, void* stream);
int rnet_slot_memory_backward(const float* dy, const float* x, const float* slot_keys,
                              const float* slot_values, const float* proj_q,
                              const float* proj_out, const float* q_cache,
                              const float* scores_cache, const int* topk_idx_cache,
                              const float* topk_w_cache, float* dx, float* d_slot_keys,
                              float* d_slot_values, float* d_proj_q, float* d_proj_out,
                              int batch, int seq_len, int dim, int n_slots, int top_k,
                              void* stream);
int rnet_swiglu_forward(const float* x, float* y, const float* gate_w, const float* up_w,
                        const float* down_w, float* gate_cache, float* up_cache, int batch_seq,
                        int dim, int d_ff, void* stream);
int rnet_swiglu_backward(const float* dy, const float* x, const float* gate_w,
                         const float* up_w, const float* down_w, const float* gate_cache,
                         const float* up_cache, float* dx, float* d_gate_w, float* d_up_w,
                         float* d_down_w, int batch_seq, int dim, int d_ff, void* stream);
int rnet_cross_entropy_forward(const float* logits, const int* targets, float* loss,
                               float* dlogits, int batch_seq, int vocab, void* stream);
/* Same result as rnet_cross_entropy_forward, but allocates nothing: for
 * callers that cannot allocate device memory while they run (a framework that
 * owns all device memory through its own pool, or a context where a
 * cudaMalloc/cudaMallocAsync is not allowed). No counterpart in the reference.
 * Scratch is a fixed 256 KiB array inside the library's device image, held on
 * every GPU that loads the library until exit, which limits batch_seq to
 * 524,280 tokens (larger sizes return RNET_ERR_ARG). The first call on each
 * device looks up that array's device address; make that first call before
 * any stream capture. All calls share the array, so calls that overlap on the
 * GPU (different streams, no ordering between them) race; calls ordered on
 * one stream are safe. The address is cached per device, so do not use this
 * entry point on a device after cudaDeviceReset. Out-of-range targets are
 * clamped to class 0 without
 * setting the device error word. */
int rnet_cross_entropy_forward_noalloc(const float* logits, const int* targets, float* loss,
                                       float* dlogits, int batch_seq, int vocab, void* stream);
int rnet_residual_add(float* x, const float* y, size_t n, void* stream);
int rnet_scale_grads(float* grads, float scale, size_t n, void* stream);

/* ------------------------------------------------------------------ data
 * Training batches of the reference's DataLoader (src/data_loader.cpp:31-52
 * as driven by src/main.cpp:117-133) with the corpus resident on the GPU.
 * rnet_data_create uploads n corpus bytes once (n = 0: the reference's
 * synthetic tokens); seed seeds the std::mt19937 the reference's training
 * loop passes to get_batch (42 + rank * 10007 there). rnet_data_batch makes
 * the reference's draws on the host (window starts, 8 bytes per sequence)
 * and gathers the windows into device int32 inputs / targets [batch *
 * seq_len] on `stream`, asynchronously; the batches equal the reference
 * loader's byte for byte. Not thread-safe per handle. */
typedef struct rnet_data rnet_data;
int rnet_data_create(const unsigned char* host_bytes, size_t n, int device, unsigned seed,
                     rnet_data** out);
int rnet_data_destroy(rnet_data* d);
int rnet_data_batch(rnet_data* d, int batch, int seq_len, int* d_inputs, int* d_targets,
                    void* stream);

/* ------------------------------------------------------------------ model
 * The reference's ResonanceNet class (include/resonance_net.h:56-130).
 * Parameters and gradients are single flat fp32 device buffers in checkpoint
 * tensor order (embed, output, final_norm, then per layer norm1..4, conv3,
 * conv7, conv15, mix, Wz, Wh, bz, bh, slot_keys, slot_values, proj_q,
 * proj_out, gate, up, down). */
typedef struct rnet_model_config {
  int d_model, n_layers, d_ff, n_heads, gru_dim, n_slots, slot_top_k, vocab_size, seq_len;
  float rms_eps;
} rnet_model_config; /* byte-identical to the 40-byte checkpoint header */

typedef struct rnet_model rnet_model;
typedef struct rnet_dist rnet_dist;

/* reference_init = 1: the reference's own initialisation (seeded uniform
 * Xavier, norm gains 1, biases 0); 0: all parameters zero. */
int rnet_model_create(const rnet_model_config* cfg, int device, int reference_init,
                      rnet_model** out);
/* Create a model from a checkpoint file (config read from its header). */
int rnet_model_create_from_checkpoint(const char* path, int device, rnet_model** out);
int rnet_model_destroy(rnet_model* m);
int rnet_model_get_config(const rnet_model* m, rnet_model_config* out);
int rnet_model_param_count(const rnet_model* m, size_t* n);
int rnet_model_device_buffers(rnet_model* m, float** d_params, float** d_grads);
int rnet_model_stream(rnet_model* m, void** stream);
int rnet_model_set_params(rnet_model* m, const float* host, size_t n);
/* Same as rnet_model_set_params from a device buffer (any stream order: the
 * call synchronises the model's stream). No counterpart in the reference. */
int rnet_model_set_params_device(rnet_model* m, const float* d_params, size_t n);
int rnet_model_get_params(rnet_model* m, float* host, size_t n);
int rnet_model_get_grads(rnet_model* m, float* host, size_t n);
/* Re-derive internal layouts after the caller wrote d_params directly. */
int rnet_model_params_updated(rnet_model* m);
int rnet_model_set_conv_quirk(rnet_model* m, int on);
/* GEMM arithmetic of the model: 0 = fp32-accurate (3xTF32 tcgen05, default),
 * 1 = bf16: every GEMM of the train step reads bf16 operands from memory
 * (tcgen05 kind::f16, fp32 accumulation): a bf16 shadow of the fp32 master
 * weights that the SGD update rewrites, and bf16 copies of the activations
 * and gradients that feed GEMMs, written by their producers. Master weights,
 * gradients, norms, scan, conv, slot selection and the optimizer stay fp32.
 * Parity with fp32 within 2e-2. */
int rnet_model_set_precision(rnet_model* m, int precision);
/* Activation recompute (no counterpart in the reference): 1 = keep only each
 * layer's input from the forward and recompute the layer's caches right
 * before its backward (one layer of caches resident instead of n_layers, at
 * the cost of one more forward per step); results are unchanged. With it on,
 * rnet_model_topk is unavailable. Default 0. */
int rnet_model_set_recompute(rnet_model* m, int on);
/* Optimizer extensions (no counterpart in the reference, whose step is plain
 * SGD with global-norm clipping; all three default to off, which keeps that
 * step): momentum (v = momentum * v + g, p -= lr * v), weight decay (wd * p
 * added to the clipped gradient) and a linear learning-rate warmup
 * (lr * min(1, (t + 1) / warmup_steps) at the t-th step after this call; the
 * reference parses TrainConfig::warmup_steps but never applies it). Resets
 * the step count and the velocity. */
int rnet_model_set_optimizer(rnet_model* m, float momentum, float weight_decay,
                             int warmup_steps);
int rnet_model_forward(rnet_model* m, const int* d_tokens, float* d_logits, int batch,
                       int seq_len);
int rnet_model_backward(rnet_model* m, const float* d_dlogits, const int* d_tokens, int batch,
                        int seq_len);
int rnet_model_zero_grad(rnet_model* m);
int rnet_model_step(rnet_model* m, float lr, float grad_clip);
/* zero_grad + forward + cross-entropy (dlogits scaled by 1/(batch*seq_len))
 * + backward + (all-reduce) + clipped SGD, all on the model stream.
 * d_loss_sum (device, may be NULL) receives the summed token loss. Without a
 * data-parallel group, repeated calls with the same batch, seq_len, lr,
 * grad_clip and model configuration replay a CUDA graph of the step captured
 * on the second such call (RNET_TRAIN_GRAPH=0 in the environment at model
 * creation keeps every step eager); the tokens are copied first, so the
 * buffers may differ from call to call. */
int rnet_model_train_step(rnet_model* m, const int* d_inputs, const int* d_targets, int batch,
                          int seq_len, float lr, float grad_clip, float* d_loss_sum);
/* Same with host token buffers; copies in, steps, copies the loss sum out and
 * waits for it. */
int rnet_model_train_step_host(rnet_model* m, const int* h_inputs, const int* h_targets,
                               int batch, int seq_len, float lr, float grad_clip,
                               float* h_loss_sum);
/* Device pointers to the last cached forward's top-k indices / weights of a
 * layer ([batch*seq_len, top_k], reference slot order). */
int rnet_model_topk(rnet_model* m, int layer, const int** d_idx, const float** d_w);
/* Host copies of the same ([batch*seq_len*top_k] each; waits for the stream). */
int rnet_model_topk_host(rnet_model* m, int layer, int* h_idx, float* h_w, size_t n);
int rnet_model_save(rnet_model* m, const char* path);
/* Checkpoint without stalling training (no counterpart in the reference,
 * whose save() blocks on a device-to-host copy): the parameters are
 * snapshotted on the model stream (a device copy ordered after all queued
 * work, so a later SGD step cannot change what is saved), then copied to
 * pinned host memory on a side stream and written by a host thread in the
 * reference byte layout. rnet_model_save_wait joins the write and returns
 * its status; a second save_async first waits for the previous one. Costs
 * one parameter-sized device buffer and one pinned host buffer. */
int rnet_model_save_async(rnet_model* m, const char* path);
int rnet_model_save_wait(rnet_model* m);
int rnet_model_load_weights(rnet_model* m, const char* path);
/* Wait for the model stream and report any device error word bits. */
int rnet_model_synchronize(rnet_model* m);

/* Per-kernel-class timing with CUDA events on the model stream. Classes
 * (index order): gemm, scan_fwd, scan_bwd, conv_fwd, conv_bwd, rms_fwd,
 * rms_bwd, slot_gather, slot_sparse_bwd, embed, cross_entropy, sgd, other.
 * read() fills arrays of n_kinds entries: total ms, algorithmic FLOPs and
 * bytes, number of timed launch groups; reset clears the record. */
#define RNET_PROFILE_KINDS 13
int rnet_model_profile_enable(rnet_model* m, int on);
int rnet_model_profile_read(rnet_model* m, double* ms, double* flops, double* bytes,
                            long long* launches, int n_kinds, int reset);

/* ------------------------------------------------------------------ decode
 * Recurrent inference with the O(1) per-stream state (per layer: the last 14
 * causal-conv inputs and the MinGRU h; 15 * d_model floats per layer per
 * stream). n_streams advance in lock step. The reference has no counterpart
 * (its `generate()` is declared, never defined; `infer` recomputes the whole
 * prefix per token). */
typedef struct rnet_decoder rnet_decoder;
int rnet_decoder_create(rnet_model* m, int n_streams, rnet_decoder** out);
int rnet_decoder_destroy(rnet_decoder* d);
/* d_tokens [n_streams, seq_len] (device). Runs the chunked-scan forward and
 * keeps the state; the last-position logits / argmax become available. Also
 * folds the slot keys / values with proj_q / proj_out for the decode steps,
 * from the weights of this moment: prefill again after changing weights. */
int rnet_decoder_prefill(rnet_decoder* d, const int* d_tokens, int seq_len);
/* One token per stream: d_tokens [n_streams] (device) or NULL to feed back
 * the previous argmax. */
int rnet_decoder_step(rnet_decoder* d, const int* d_tokens);
/* n_steps greedy steps (fed back on the device); d_out [n_steps, n_streams]
 * (device, may be NULL). use_graph = 1 replays one captured CUDA graph per step. */
int rnet_decoder_generate(rnet_decoder* d, int n_steps, int* d_out, int use_graph);
/* Next-token rule of prefill / step / generate: temperature <= 0 = greedy
 * argmax (default); otherwise the reference infer loop's temperature + top-p
 * sampling (src/main.cpp:327-360: softmax at `temperature`, probabilities
 * sorted descending, smallest prefix reaching `top_p`, sample within it),
 * computed on the device. The uniform for stream m at the sampled token's
 * position pos is a splitmix64 hash of (seed, m, pos), so runs are
 * reproducible and independent of batching; it is not the reference CLI's
 * std::mt19937 stream. Ties in probability order by token id. */
int rnet_decoder_set_sampling(rnet_decoder* d, float temperature, float top_p,
                              unsigned long long seed);
/* Device pointers to the current logits [n_streams, vocab] and next tokens
 * [n_streams], and the state buffer with its size per stream in floats. */
int rnet_decoder_outputs(rnet_decoder* d, const float** d_logits, const int** d_next);
/* Host copies of the same (either pointer may be NULL); waits for the stream. */
int rnet_decoder_outputs_host(rnet_decoder* d, float* h_logits, int* h_next);
int rnet_decoder_state(rnet_decoder* d, float** d_state, size_t* floats_per_stream);

/* ------------------------------------------------------------------ data parallel
 * The reference's include/dist.h:12-36 over NCCL (loaded at run time). */
int rnet_dist_unique_id(unsigned char uid[128]);
int rnet_dist_create(int rank, int world, int local_rank, const unsigned char uid[128],
                     int timeout_ms, rnet_dist** out);
int rnet_dist_destroy(rnet_dist* d);
int rnet_dist_allreduce_sum(rnet_dist* d, float* d_buf, size_t count, void* stream);
int rnet_dist_group_start(rnet_dist* d);
int rnet_dist_group_end(rnet_dist* d);
/* File rendezvous of the 128-byte unique id (reference src/dist.cpp:53-93):
 * write = write "<path>.tmp" then rename (readers never see a partial file);
 * read = poll until a complete file appears, RNET_ERR_TIMEOUT after
 * timeout_ms, RNET_ERR_IO on a short/unreadable file. Host only. */
int rnet_dist_uid_file_write(const char* path, const unsigned char uid[128]);
int rnet_dist_uid_file_read(const char* path, int timeout_ms, unsigned char uid[128]);
/* Attach (or detach with NULL): backward then all-reduces gradient buckets
 * as they complete and step() uses the reference's world-size scaling. */
int rnet_model_set_dist(rnet_model* m, rnet_dist* d);

#ifdef __cplusplus
}
#endif

#endif /* RNET_CAPI_H */
