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

/* Read (and optionally clear) the device error word of the current device:
 * bit 0 = a bounded wait timed out, bit 1 = out-of-range index seen,
 * bit 2 = TMEM allocation failed. Synchronises the device. */
int rnet_device_error(unsigned* word, int clear);

/* ------------------------------------------------------------------ GEMM engine
 * C[M,N] (op)= alpha * A[M,K] * B[N,K]^T on the tcgen05 3xTF32 engine.
 * a_mn_major = 0: A(i,k) = A[i*lda + k]; 1: A(i,k) = A[k*lda + i]  (same for B).
 * op: 0 = store, 1 = accumulate (C += ...), 2 = residual (C = R + ...).
 * lda/ldb must be multiples of 4 and A/B 16-byte aligned. */
int rnet_gemm_f32(int M, int N, int K, const float* A, int lda, int a_mn_major, const float* B,
                  int ldb, int b_mn_major, float* C, int ldc, const float* R, int ldr, int op,
                  float alpha, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RNET_CAPI_H */
