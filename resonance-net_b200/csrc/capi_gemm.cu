// C-ABI entry of the GEMM engine (used by parity tests and by callers that
// want the engine directly).
#include <string>

#include "gemm.cuh"
#include "status.h"

static int g_gemm_precision = 0;

extern "C" int rnet_gemm_set_precision(int precision) {
  if (precision != 0 && precision != 1)
    return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_set_precision: expected 0 or 1");
  g_gemm_precision = precision;
  return RNET_OK;
}

extern "C" int rnet_gemm_f32(int M, int N, int K, const float* A, int lda, int a_mn_major,
                             const float* B, int ldb, int b_mn_major, float* C, int ldc,
                             const float* R, int ldr, int op, float alpha, void* stream) {
  using namespace rnet_gemm;
  if (op < 0 || op > 2) return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_f32: bad op");
  if (op == 2 && R == nullptr) return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_f32: null R");
  Operand a{A, lda, a_mn_major != 0};
  Operand b{B, ldb, b_mn_major != 0};
  Epilogue e;
  e.kind = op == 0 ? EPI_STORE : (op == 1 ? EPI_ACCUM : EPI_RESID);
  e.alpha = alpha;
  e.C = C;
  e.ldc = ldc;
  e.R = R;
  e.ldr = ldr;
  cudaError_t err = gemm_tf32x3((cudaStream_t)stream, M, N, K, a, b, e, 0, 0,
                                rnet_status::device_error_word(), g_gemm_precision);
  if (err != cudaSuccess) {
    const std::string what = std::string("rnet_gemm_f32 (") + gemm_last_reason() + ")";
    return rnet_status::fail_cuda(err, what.c_str());
  }
  return RNET_OK;
}

extern "C" int rnet_gemm_set_cta_group(int cta_group) {
  if (cta_group < 0 || cta_group > 2)
    return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_set_cta_group: expected 0, 1 or 2");
  rnet_gemm::set_force_cta_group(cta_group);
  return RNET_OK;
}

extern "C" int rnet_gemm_bf16(int M, int N, int K, const void* A, int lda, int a_mn_major,
                              const void* B, int ldb, int b_mn_major, float* C, int ldc,
                              const float* R, int ldr, int op, float alpha, void* C16,
                              void* stream) {
  using namespace rnet_gemm;
  if (op < 0 || op > 2) return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_bf16: bad op");
  if (op == 2 && R == nullptr) return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_bf16: null R");
  if (op == 1 && C16) return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_bf16: C16 with op 1");
  Operand a = bf16_operand(static_cast<const __nv_bfloat16*>(A), lda, a_mn_major != 0);
  Operand b = bf16_operand(static_cast<const __nv_bfloat16*>(B), ldb, b_mn_major != 0);
  Epilogue e;
  e.kind = op == 0 ? EPI_STORE : (op == 1 ? EPI_ACCUM : EPI_RESID);
  e.alpha = alpha;
  e.C = C;
  e.ldc = ldc;
  e.R = R;
  e.ldr = ldr;
  e.C16 = static_cast<__nv_bfloat16*>(C16);
  if (e.C16 && (ldc % 8 || (reinterpret_cast<uintptr_t>(C16) & 15)))
    return rnet_status::fail(RNET_ERR_ARG, "rnet_gemm_bf16: C16 needs 16-byte aligned rows");
  cudaError_t err = gemm_tf32x3((cudaStream_t)stream, M, N, K, a, b, e, 0, 0,
                                rnet_status::device_error_word(), PREC_TF32X3);
  if (err != cudaSuccess) {
    const std::string what = std::string("rnet_gemm_bf16 (") + gemm_last_reason() + ")";
    return rnet_status::fail_cuda(err, what.c_str());
  }
  return RNET_OK;
}
