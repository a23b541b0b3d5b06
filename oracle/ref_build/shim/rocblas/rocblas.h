// TEST INFRASTRUCTURE.  The slice of the rocBLAS API that the reference's
// csrc/nova_winograd.hip calls, mapped onto cuBLAS, so the reference's host
// class (set_weights, forward, forward_workspace) runs unchanged on a CUDA GPU.
// rocBLAS's gemm_strided_batched_ex contract -- column-major
// D = alpha*op(A)*op(B) + beta*C per batch, FP16 operands, FP32 compute, FP16
// result -- is cuBLAS's cublasGemmStridedBatchedEx with CUBLAS_COMPUTE_32F.
// Only C == D (in place), as the reference passes, is supported.
#pragma once
#include <cstdint>
#include <cublas_v2.h>
#include <cuda_runtime.h>

typedef cublasHandle_t rocblas_handle;
typedef int rocblas_status;
typedef long long rocblas_stride;
enum { rocblas_status_success = 0, rocblas_status_not_implemented = 2 };
typedef enum { rocblas_operation_none = 111, rocblas_operation_transpose = 112 } rocblas_operation;
typedef enum { rocblas_datatype_f16_r = 150, rocblas_datatype_f32_r = 151 } rocblas_datatype;
typedef enum { rocblas_gemm_algo_standard = 0 } rocblas_gemm_algo;

inline rocblas_status rocblas_create_handle(rocblas_handle* h) { return (int)cublasCreate(h); }
inline rocblas_status rocblas_destroy_handle(rocblas_handle h) { return (int)cublasDestroy(h); }
inline rocblas_status rocblas_set_stream(rocblas_handle h, cudaStream_t s) {
  return (int)cublasSetStream(h, s);
}

inline cudaDataType_t nova_ref_dtype(rocblas_datatype t) {
  return t == rocblas_datatype_f16_r ? CUDA_R_16F : CUDA_R_32F;
}

inline rocblas_status rocblas_gemm_strided_batched_ex(
    rocblas_handle h, rocblas_operation ta, rocblas_operation tb, int m, int n, int k,
    const void* alpha, const void* a, rocblas_datatype at, int lda, rocblas_stride sa,
    const void* b, rocblas_datatype bt, int ldb, rocblas_stride sb, const void* beta, const void* c,
    rocblas_datatype ct, int ldc, rocblas_stride sc, void* d, rocblas_datatype dt, int ldd,
    rocblas_stride sd, int batch, rocblas_datatype compute, rocblas_gemm_algo, int32_t, uint32_t) {
  if (c != d || ct != dt || ldc != ldd || sc != sd || compute != rocblas_datatype_f32_r)
    return rocblas_status_not_implemented;
  const cublasOperation_t oa = ta == rocblas_operation_none ? CUBLAS_OP_N : CUBLAS_OP_T;
  const cublasOperation_t ob = tb == rocblas_operation_none ? CUBLAS_OP_N : CUBLAS_OP_T;
  return (int)cublasGemmStridedBatchedEx(h, oa, ob, m, n, k, alpha, a, nova_ref_dtype(at), lda, sa,
                                         b, nova_ref_dtype(bt), ldb, sb, beta, d,
                                         nova_ref_dtype(dt), ldd, sd, batch, CUBLAS_COMPUTE_32F,
                                         CUBLAS_GEMM_DEFAULT);
}
