/*
 * cfi_cublas.h -- cuBLAS-compatible dense GEMM entry points of libcfi_b200.so (sm_100a).
 *
 * Same argument meaning, column-major semantics and status codes as the cuBLAS calls they stand
 * in for (cuda-for-intel crates/cublas_shim/src/lib.rs:887-1076, validation plan.rs:160-215):
 * C = alpha * op(A) * op(B) + beta * C.  f16/bf16 inputs with op(A) = A^T and op(B) = B -- the
 * layout ggml uses for its dense and attention GEMMs -- run on the 5th-generation tensor cores
 * (tcgen05, fp32 accumulate in tensor memory, TMA-fed) -- or, with at most 8 columns (decode-time
 * attention), a warp-per-row skinny kernel; every other legal combination runs a SIMT kernel with
 * fp32 accumulation.  Calls are asynchronous on the handle's stream.
 */
#ifndef CFI_CUBLAS_H
#define CFI_CUBLAS_H
#include <stddef.h>
#include <stdint.h>

#ifndef CFI_API
#define CFI_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* cublasStatus_t values */
enum {
    CFI_BLAS_SUCCESS = 0,
    CFI_BLAS_NOT_INITIALIZED = 1,
    CFI_BLAS_ALLOC_FAILED = 3,
    CFI_BLAS_INVALID_VALUE = 7,
    CFI_BLAS_EXECUTION_FAILED = 13,
    CFI_BLAS_NOT_SUPPORTED = 15
};
/* cublasOperation_t, cudaDataType_t, cublasComputeType_t, cublasPointerMode_t values */
enum { CFI_OP_N = 0, CFI_OP_T = 1, CFI_OP_C = 2 };
enum { CFI_R_32F = 0, CFI_R_16F = 2, CFI_R_16BF = 14 };
enum { CFI_COMPUTE_16F = 64, CFI_COMPUTE_32F = 68, CFI_COMPUTE_32F_FAST_16F = 74, CFI_COMPUTE_32F_FAST_16BF = 75,
       CFI_COMPUTE_32F_FAST_TF32 = 77 };
enum { CFI_POINTER_MODE_HOST = 0, CFI_POINTER_MODE_DEVICE = 1 };

typedef struct cfi_blas cfi_blas;

/* cublasCreate_v2 / cublasDestroy_v2 (lib.rs handle state) */
CFI_API int cfi_blas_create(cfi_blas **handle);
CFI_API int cfi_blas_destroy(cfi_blas *handle);
/* cublasSetStream_v2 / cublasGetStream_v2 */
CFI_API int cfi_blas_set_stream(cfi_blas *handle, void *stream);
CFI_API int cfi_blas_get_stream(cfi_blas *handle, void **stream);
/* cublasSetPointerMode_v2: alpha/beta read from host (0) or device (1) memory */
CFI_API int cfi_blas_set_pointer_mode(cfi_blas *handle, int mode);

/* cublasGemmEx (lib.rs:887-929) */
CFI_API int cfi_blas_gemm_ex(cfi_blas *handle, int transa, int transb, int m, int n, int k, const void *alpha,
                             const void *A, int a_type, int lda, const void *B, int b_type, int ldb, const void *beta,
                             void *C, int c_type, int ldc, int compute_type, int algo);
/* cublasGemmStridedBatchedEx (lib.rs:932-985); strides in elements */
CFI_API int cfi_blas_gemm_strided_batched_ex(cfi_blas *handle, int transa, int transb, int m, int n, int k,
                                             const void *alpha, const void *A, int a_type, int lda, long long stride_a,
                                             const void *B, int b_type, int ldb, long long stride_b, const void *beta,
                                             void *C, int c_type, int ldc, long long stride_c, int batch_count,
                                             int compute_type, int algo);
/* cublasGemmBatchedEx (lib.rs:988-1034): device arrays of per-batch pointers */
CFI_API int cfi_blas_gemm_batched_ex(cfi_blas *handle, int transa, int transb, int m, int n, int k, const void *alpha,
                                     const void *const A[], int a_type, int lda, const void *const B[], int b_type,
                                     int ldb, const void *beta, void *const C[], int c_type, int ldc, int batch_count,
                                     int compute_type, int algo);
/* cublasSgemm_v2 (lib.rs:1037-1076) */
CFI_API int cfi_blas_sgemm(cfi_blas *handle, int transa, int transb, int m, int n, int k, const float *alpha,
                           const float *A, int lda, const float *B, int ldb, const float *beta, float *C, int ldc);

/* plan::validate (plan.rs:160-215): 0, CFI_BLAS_INVALID_VALUE or CFI_BLAS_NOT_SUPPORTED. */
CFI_API int cfi_blas_validate(int transa, int transb, int m, int n, int k, int lda, int ldb, int ldc, int a_type,
                              int b_type, int c_type, int compute_type);
/* Which kernel the last GEMM call of this handle ran: 1 tcgen05, 2 SIMT, 3 skinny (n <= 8 columns),
 * 0 none (early return). */
CFI_API int cfi_blas_last_path(cfi_blas *handle);

#ifdef __cplusplus
}
#endif
#endif
