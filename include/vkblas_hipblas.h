/* vkblas_hipblas.h -- hipBLAS / rocBLAS ABI surface of libvkblas_hipblas.so.
 *
 * Drop-in for the LD_PRELOAD shim of lakitu12/vkblas (src/vkblas_hipblas.c).
 * No HIP or ROCm headers exist on a CUDA machine, so the ABI types are
 * declared here.  Enum values follow the public hipBLAS / rocBLAS / HIP
 * headers; the ones the reference itself spells out are cited, the others are
 * marked "public header value".
 *
 * Semantics kept from the reference:
 *   - column-major hipBLAS arguments are translated to the row-major engine
 *     by swapping operands (src/vkblas_hipblas.c:234-239): op_a <- transB,
 *     op_b <- transA, M <- n, N <- m, A <- B, B <- A;
 *   - m, n, k <= 0 (and batchCount <= 0) return INVALID_VALUE, a NULL handle
 *     returns INVALID_VALUE (src/vkblas_hipblas.c:223, 257, 406);
 *   - fp32 via hipblasSgemm / _v2 Ex / rocblas; fp16 and bf16 when A, B and C
 *     all carry that type (src/vkblas_hipblas.c:276-284, 417-466);
 *   - anything not handled is forwarded by dlsym to the real library; when
 *     the real library is absent (every CUDA machine), the call returns
 *     HIPBLAS_STATUS_NOT_SUPPORTED (src/vkblas_hipblas.c:62-65) or
 *     rocblas_status_not_implemented (src/vkblas_hipblas.c:821-824).
 *
 * Differences from the reference:
 *   - handles are this library's own objects holding stream, pointer mode and
 *     (when a real hipBLAS exists) the real handle used for forwarding; the
 *     reference kept stream and pointer mode in process globals;
 *   - calls are stream-ordered on the handle's stream (a hipStream_t is a
 *     cudaStream_t here); no host synchronisation is made before or after;
 *   - with HIPBLAS_POINTER_MODE_DEVICE the kernels read alpha/beta from device
 *     memory themselves instead of a blocking device-to-host copy
 *     (src/vkblas_hipblas.c:126-131).
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ HIP types */
typedef struct ihipStream_t* hipStream_t;      /* == cudaStream_t on CUDA */
typedef int hipError_t;
typedef struct { float x, y; } hipComplex;
typedef struct { double x, y; } hipDoubleComplex;

typedef enum {                                 /* public header values */
    HIP_R_32F = 0, HIP_R_64F = 1, HIP_R_16F = 2, HIP_R_8I = 3,
    HIP_C_32F = 4, HIP_C_64F = 5, HIP_C_16F = 6, HIP_C_8I = 7,
    HIP_R_8U = 8, HIP_C_8U = 9, HIP_R_32I = 10, HIP_C_32I = 11,
    HIP_R_32U = 12, HIP_C_32U = 13, HIP_R_16BF = 14, HIP_C_16BF = 15
} hipDataType;                                 /* R_16F=2, R_16BF=14: src/vkblas_hipblas.c:280 */

/* --------------------------------------------------------- hipBLAS types */
typedef void* hipblasHandle_t;
typedef int64_t hipblasStride;

typedef enum {                                 /* public header values */
    HIPBLAS_STATUS_SUCCESS = 0,
    HIPBLAS_STATUS_NOT_INITIALIZED = 1,
    HIPBLAS_STATUS_ALLOC_FAILED = 2,
    HIPBLAS_STATUS_INVALID_VALUE = 3,
    HIPBLAS_STATUS_MAPPING_ERROR = 4,
    HIPBLAS_STATUS_EXECUTION_FAILED = 5,
    HIPBLAS_STATUS_INTERNAL_ERROR = 6,
    HIPBLAS_STATUS_NOT_SUPPORTED = 7,
    HIPBLAS_STATUS_ARCH_MISMATCH = 8,
    HIPBLAS_STATUS_HANDLE_IS_NULLPTR = 9,
    HIPBLAS_STATUS_INVALID_ENUM = 10,
    HIPBLAS_STATUS_UNKNOWN = 11
} hipblasStatus_t;

typedef enum { HIPBLAS_OP_N = 111, HIPBLAS_OP_T = 112, HIPBLAS_OP_C = 113 } hipblasOperation_t;
typedef enum { HIPBLAS_POINTER_MODE_HOST = 0, HIPBLAS_POINTER_MODE_DEVICE = 1 } hipblasPointerMode_t;
typedef enum { HIPBLAS_ATOMICS_NOT_ALLOWED = 0, HIPBLAS_ATOMICS_ALLOWED = 1 } hipblasAtomicsMode_t;
typedef enum { HIPBLAS_FILL_MODE_UPPER = 121, HIPBLAS_FILL_MODE_LOWER = 122,
               HIPBLAS_FILL_MODE_FULL = 123 } hipblasFillMode_t;
typedef enum { HIPBLAS_DIAG_NON_UNIT = 131, HIPBLAS_DIAG_UNIT = 132 } hipblasDiagType_t;
typedef enum { HIPBLAS_SIDE_LEFT = 141, HIPBLAS_SIDE_RIGHT = 142,
               HIPBLAS_SIDE_BOTH = 143 } hipblasSideMode_t;

/* Legacy hipblasDatatype_t (R_16F=150, R_16B=168: src/vkblas_hipblas.c:280-284). */
typedef enum {
    HIPBLAS_R_16F = 150, HIPBLAS_R_32F = 151, HIPBLAS_R_64F = 152,
    HIPBLAS_C_16F = 153, HIPBLAS_C_32F = 154, HIPBLAS_C_64F = 155,
    HIPBLAS_R_8I = 160, HIPBLAS_R_8U = 161, HIPBLAS_R_32I = 162, HIPBLAS_R_32U = 163,
    HIPBLAS_C_8I = 164, HIPBLAS_C_8U = 165, HIPBLAS_C_32I = 166, HIPBLAS_C_32U = 167,
    HIPBLAS_R_16B = 168, HIPBLAS_C_16B = 169
} hipblasDatatype_t;

typedef enum {                                 /* public header values */
    HIPBLAS_COMPUTE_16F = 0, HIPBLAS_COMPUTE_16F_PEDANTIC = 1,
    HIPBLAS_COMPUTE_32F = 2, HIPBLAS_COMPUTE_32F_PEDANTIC = 3,
    HIPBLAS_COMPUTE_32F_FAST_16F = 4, HIPBLAS_COMPUTE_32F_FAST_16BF = 5,
    HIPBLAS_COMPUTE_32F_FAST_TF32 = 6, HIPBLAS_COMPUTE_64F = 7,
    HIPBLAS_COMPUTE_64F_PEDANTIC = 8, HIPBLAS_COMPUTE_32I = 9,
    HIPBLAS_COMPUTE_32I_PEDANTIC = 10
} hipblasComputeType_t;

typedef enum { HIPBLAS_GEMM_DEFAULT = 160 } hipblasGemmAlgo_t;  /* public header value */

/* The legacy hipblasGemmEx carries its compute type as a hipblasDatatype_t in
 * older headers and a hipblasComputeType_t in newer ones
 * (src/vkblas_hipblas.c:19-35); both are a 32-bit int at the ABI. */
typedef int vkblas_gemmex_compute_t;

/* --------------------------------------------------------- rocBLAS types */
typedef struct _rocblas_handle* rocblas_handle;
typedef int32_t rocblas_int;
typedef int64_t rocblas_stride;
typedef enum {                                 /* public header values */
    rocblas_status_success = 0, rocblas_status_invalid_handle = 1,
    rocblas_status_not_implemented = 2, rocblas_status_invalid_pointer = 3,
    rocblas_status_invalid_size = 4, rocblas_status_memory_error = 5,
    rocblas_status_internal_error = 6, rocblas_status_perf_degraded = 7,
    rocblas_status_size_query_mismatch = 8, rocblas_status_size_increased = 9,
    rocblas_status_size_unchanged = 10, rocblas_status_invalid_value = 11,
    rocblas_status_continue = 12, rocblas_status_check_numerics_fail = 13
} rocblas_status;
typedef enum { rocblas_operation_none = 111, rocblas_operation_transpose = 112,
               rocblas_operation_conjugate_transpose = 113 } rocblas_operation;
typedef enum {                                 /* f32_r = 151: src/vkblas_hipblas.c:839 */
    rocblas_datatype_f16_r = 150, rocblas_datatype_f32_r = 151, rocblas_datatype_f64_r = 152,
    rocblas_datatype_f16_c = 153, rocblas_datatype_f32_c = 154, rocblas_datatype_f64_c = 155,
    rocblas_datatype_i8_r = 160, rocblas_datatype_u8_r = 161, rocblas_datatype_i32_r = 162,
    rocblas_datatype_u32_r = 163, rocblas_datatype_i8_c = 164, rocblas_datatype_u8_c = 165,
    rocblas_datatype_i32_c = 166, rocblas_datatype_u32_c = 167,
    rocblas_datatype_bf16_r = 168, rocblas_datatype_bf16_c = 169
} rocblas_datatype;
typedef enum { rocblas_gemm_algo_standard = 0 } rocblas_gemm_algo;
typedef enum { rocblas_pointer_mode_host = 0, rocblas_pointer_mode_device = 1 } rocblas_pointer_mode;

/* ------------------------------------------------ handle management
 * reference src/vkblas_hipblas.c:69-123 */
hipblasStatus_t hipblasCreate(hipblasHandle_t* handle);
hipblasStatus_t hipblasDestroy(hipblasHandle_t handle);
hipblasStatus_t hipblasSetStream(hipblasHandle_t handle, hipStream_t streamId);
hipblasStatus_t hipblasGetStream(hipblasHandle_t handle, hipStream_t* streamId);
hipblasStatus_t hipblasSetPointerMode(hipblasHandle_t handle, hipblasPointerMode_t mode);
hipblasStatus_t hipblasGetPointerMode(hipblasHandle_t handle, hipblasPointerMode_t* mode);
hipblasStatus_t hipblasSetAtomicsMode(hipblasHandle_t handle, hipblasAtomicsMode_t atomics_mode);
hipblasStatus_t hipblasSetWorkspace(hipblasHandle_t handle, void* workspace, size_t size);
hipblasStatus_t hipblasGetVersion(hipblasHandle_t handle, int* version);
const char* hipblasStatusToString(hipblasStatus_t status);

/* ------------------------------------------------ intercepted GEMMs
 * reference src/vkblas_hipblas.c:403-466 */
hipblasStatus_t hipblasSgemm(hipblasHandle_t handle, hipblasOperation_t transA,
                             hipblasOperation_t transB, int m, int n, int k, const float* alpha,
                             const float* AP, int lda, const float* BP, int ldb,
                             const float* beta, float* CP, int ldc);
hipblasStatus_t hipblasSgemmStridedBatched(hipblasHandle_t handle, hipblasOperation_t transA,
                                           hipblasOperation_t transB, int m, int n, int k,
                                           const float* alpha, const float* AP, int lda,
                                           long long strideA, const float* BP, int ldb,
                                           long long strideB, const float* beta, float* CP,
                                           int ldc, long long strideC, int batchCount);
hipblasStatus_t hipblasGemmEx_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                 hipblasOperation_t transB, int m, int n, int k,
                                 const void* alpha, const void* A, hipDataType aType, int lda,
                                 const void* B, hipDataType bType, int ldb, const void* beta,
                                 void* C, hipDataType cType, int ldc,
                                 hipblasComputeType_t computeType, hipblasGemmAlgo_t algo);
hipblasStatus_t hipblasGemmStridedBatchedEx_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                               hipblasOperation_t transB, int m, int n, int k,
                                               const void* alpha, const void* A,
                                               hipDataType aType, int lda, hipblasStride strideA,
                                               const void* B, hipDataType bType, int ldb,
                                               hipblasStride strideB, const void* beta, void* C,
                                               hipDataType cType, int ldc, hipblasStride strideC,
                                               int batchCount, hipblasComputeType_t computeType,
                                               hipblasGemmAlgo_t algo);
hipblasStatus_t hipblasGemmEx(hipblasHandle_t handle, hipblasOperation_t transA,
                              hipblasOperation_t transB, int m, int n, int k, const void* alpha,
                              const void* A, hipblasDatatype_t aType, int lda, const void* B,
                              hipblasDatatype_t bType, int ldb, const void* beta, void* C,
                              hipblasDatatype_t cType, int ldc,
                              vkblas_gemmex_compute_t computeType, hipblasGemmAlgo_t algo);

/* ---------------------------------------- fp64 / complex GEMMs
 * reference src/vkblas_hipblas.c:470-620.  Run on vkblas_gemm_{f64,c64,z64}
 * (operands swapped into the engine's row-major contract) on the handle's
 * stream; forwarded to the real library when the engine declines.  Scalars
 * in device memory (pointer mode DEVICE) are read with one blocking copy; a
 * conjugate transpose (HIPBLAS_OP_C) of a complex operand is forwarded. */
hipblasStatus_t hipblasDgemm(hipblasHandle_t handle, hipblasOperation_t transA,
                             hipblasOperation_t transB, int m, int n, int k, const double* alpha,
                             const double* AP, int lda, const double* BP, int ldb,
                             const double* beta, double* CP, int ldc);
hipblasStatus_t hipblasDgemmStridedBatched(hipblasHandle_t handle, hipblasOperation_t transA,
                                           hipblasOperation_t transB, int m, int n, int k,
                                           const double* alpha, const double* AP, int lda,
                                           long long strideA, const double* BP, int ldb,
                                           long long strideB, const double* beta, double* CP,
                                           int ldc, long long strideC, int batchCount);
hipblasStatus_t hipblasCgemm_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                hipblasOperation_t transB, int m, int n, int k,
                                const hipComplex* alpha, const hipComplex* AP, int lda,
                                const hipComplex* BP, int ldb, const hipComplex* beta,
                                hipComplex* CP, int ldc);
hipblasStatus_t hipblasCgemmStridedBatched_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                              hipblasOperation_t transB, int m, int n, int k,
                                              const hipComplex* alpha, const hipComplex* AP,
                                              int lda, long long strideA, const hipComplex* BP,
                                              int ldb, long long strideB, const hipComplex* beta,
                                              hipComplex* CP, int ldc, long long strideC,
                                              int batchCount);
hipblasStatus_t hipblasZgemm_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                hipblasOperation_t transB, int m, int n, int k,
                                const hipDoubleComplex* alpha, const hipDoubleComplex* AP, int lda,
                                const hipDoubleComplex* BP, int ldb, const hipDoubleComplex* beta,
                                hipDoubleComplex* CP, int ldc);
hipblasStatus_t hipblasZgemmStridedBatched_v2(hipblasHandle_t handle, hipblasOperation_t transA,
                                              hipblasOperation_t transB, int m, int n, int k,
                                              const hipDoubleComplex* alpha,
                                              const hipDoubleComplex* AP, int lda,
                                              long long strideA, const hipDoubleComplex* BP,
                                              int ldb, long long strideB,
                                              const hipDoubleComplex* beta, hipDoubleComplex* CP,
                                              int ldc, long long strideC, int batchCount);

/* ------------------------- forward-only BLAS-1/2/3 and LAPACK-like calls
 * reference src/vkblas_hipblas.c:632-800 (pure dlsym forwarding there too) */
hipblasStatus_t hipblasSdot(hipblasHandle_t, int, const float*, int, const float*, int, float*);
hipblasStatus_t hipblasDdot(hipblasHandle_t, int, const double*, int, const double*, int, double*);
hipblasStatus_t hipblasCdotc_v2(hipblasHandle_t, int, const hipComplex*, int, const hipComplex*,
                                int, hipComplex*);
hipblasStatus_t hipblasCdotu_v2(hipblasHandle_t, int, const hipComplex*, int, const hipComplex*,
                                int, hipComplex*);
hipblasStatus_t hipblasZdotc_v2(hipblasHandle_t, int, const hipDoubleComplex*, int,
                                const hipDoubleComplex*, int, hipDoubleComplex*);
hipblasStatus_t hipblasZdotu_v2(hipblasHandle_t, int, const hipDoubleComplex*, int,
                                const hipDoubleComplex*, int, hipDoubleComplex*);
hipblasStatus_t hipblasDotEx_v2(hipblasHandle_t, int, const void*, hipDataType, int, const void*,
                                hipDataType, int, void*, hipDataType, hipDataType);
hipblasStatus_t hipblasSgemv(hipblasHandle_t, hipblasOperation_t, int, int, const float*,
                             const float*, int, const float*, int, const float*, float*, int);
hipblasStatus_t hipblasDgemv(hipblasHandle_t, hipblasOperation_t, int, int, const double*,
                             const double*, int, const double*, int, const double*, double*, int);
hipblasStatus_t hipblasCgemv_v2(hipblasHandle_t, hipblasOperation_t, int, int, const hipComplex*,
                                const hipComplex*, int, const hipComplex*, int, const hipComplex*,
                                hipComplex*, int);
hipblasStatus_t hipblasZgemv_v2(hipblasHandle_t, hipblasOperation_t, int, int,
                                const hipDoubleComplex*, const hipDoubleComplex*, int,
                                const hipDoubleComplex*, int, const hipDoubleComplex*,
                                hipDoubleComplex*, int);
hipblasStatus_t hipblasStrsm(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                             hipblasOperation_t, hipblasDiagType_t, int, int, const float*,
                             const float*, int, float*, int);
hipblasStatus_t hipblasDtrsm(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                             hipblasOperation_t, hipblasDiagType_t, int, int, const double*,
                             const double*, int, double*, int);
hipblasStatus_t hipblasCtrsm_v2(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                hipblasOperation_t, hipblasDiagType_t, int, int,
                                const hipComplex*, const hipComplex*, int, hipComplex*, int);
hipblasStatus_t hipblasZtrsm_v2(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                hipblasOperation_t, hipblasDiagType_t, int, int,
                                const hipDoubleComplex*, const hipDoubleComplex*, int,
                                hipDoubleComplex*, int);
hipblasStatus_t hipblasStrsmBatched(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                    hipblasOperation_t, hipblasDiagType_t, int, int,
                                    const float*, const float* const[], int, float* const[], int,
                                    int);
hipblasStatus_t hipblasDtrsmBatched(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                    hipblasOperation_t, hipblasDiagType_t, int, int,
                                    const double*, const double* const[], int, double* const[],
                                    int, int);
hipblasStatus_t hipblasCtrsmBatched_v2(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                       hipblasOperation_t, hipblasDiagType_t, int, int,
                                       const hipComplex*, const hipComplex* const[], int,
                                       hipComplex* const[], int, int);
hipblasStatus_t hipblasZtrsmBatched_v2(hipblasHandle_t, hipblasSideMode_t, hipblasFillMode_t,
                                       hipblasOperation_t, hipblasDiagType_t, int, int,
                                       const hipDoubleComplex*, const hipDoubleComplex* const[],
                                       int, hipDoubleComplex* const[], int, int);
hipblasStatus_t hipblasSgelsBatched(hipblasHandle_t, hipblasOperation_t, const int, const int,
                                    const int, float* const[], const int, float* const[],
                                    const int, int*, int*, const int);
hipblasStatus_t hipblasDgelsBatched(hipblasHandle_t, hipblasOperation_t, const int, const int,
                                    const int, double* const[], const int, double* const[],
                                    const int, int*, int*, const int);
hipblasStatus_t hipblasCgelsBatched_v2(hipblasHandle_t, hipblasOperation_t, const int, const int,
                                       const int, hipComplex* const[], const int,
                                       hipComplex* const[], const int, int*, int*, const int);
hipblasStatus_t hipblasZgelsBatched_v2(hipblasHandle_t, hipblasOperation_t, const int, const int,
                                       const int, hipDoubleComplex* const[], const int,
                                       hipDoubleComplex* const[], const int, int*, int*,
                                       const int);
hipblasStatus_t hipblasSgeqrfBatched(hipblasHandle_t, const int, const int, float* const[],
                                     const int, float* const[], int*, const int);
hipblasStatus_t hipblasDgeqrfBatched(hipblasHandle_t, const int, const int, double* const[],
                                     const int, double* const[], int*, const int);
hipblasStatus_t hipblasCgeqrfBatched_v2(hipblasHandle_t, const int, const int,
                                        hipComplex* const[], const int, hipComplex* const[],
                                        int*, const int);
hipblasStatus_t hipblasZgeqrfBatched_v2(hipblasHandle_t, const int, const int,
                                        hipDoubleComplex* const[], const int,
                                        hipDoubleComplex* const[], int*, const int);
hipblasStatus_t hipblasSgetrfBatched(hipblasHandle_t, const int, float* const[], const int, int*,
                                     int*, const int);
hipblasStatus_t hipblasDgetrfBatched(hipblasHandle_t, const int, double* const[], const int,
                                     int*, int*, const int);
hipblasStatus_t hipblasCgetrfBatched_v2(hipblasHandle_t, const int, hipComplex* const[],
                                        const int, int*, int*, const int);
hipblasStatus_t hipblasZgetrfBatched_v2(hipblasHandle_t, const int, hipDoubleComplex* const[],
                                        const int, int*, int*, const int);
hipblasStatus_t hipblasSgetrsBatched(hipblasHandle_t, const hipblasOperation_t, const int,
                                     const int, float* const[], const int, const int*,
                                     float* const[], const int, int*, const int);
hipblasStatus_t hipblasDgetrsBatched(hipblasHandle_t, const hipblasOperation_t, const int,
                                     const int, double* const[], const int, const int*,
                                     double* const[], const int, int*, const int);
hipblasStatus_t hipblasCgetrsBatched_v2(hipblasHandle_t, const hipblasOperation_t, const int,
                                        const int, hipComplex* const[], const int, const int*,
                                        hipComplex* const[], const int, int*, const int);
hipblasStatus_t hipblasZgetrsBatched_v2(hipblasHandle_t, const hipblasOperation_t, const int,
                                        const int, hipDoubleComplex* const[], const int,
                                        const int*, hipDoubleComplex* const[], const int, int*,
                                        const int);

/* ------------------------------------------------ rocBLAS intercepts
 * reference src/vkblas_hipblas.c:802-955.  Handled only when c == d,
 * ldc == ldd and compute_type == rocblas_datatype_f32_r (840, 904). */
rocblas_status rocblas_gemm_ex(rocblas_handle handle, rocblas_operation transA,
                               rocblas_operation transB, rocblas_int m, rocblas_int n,
                               rocblas_int k, const void* alpha, const void* a,
                               rocblas_datatype a_type, rocblas_int lda, const void* b,
                               rocblas_datatype b_type, rocblas_int ldb, const void* beta,
                               const void* c, rocblas_datatype c_type, rocblas_int ldc, void* d,
                               rocblas_datatype d_type, rocblas_int ldd,
                               rocblas_datatype compute_type, rocblas_gemm_algo algo,
                               int32_t solution_index, uint32_t flags);
rocblas_status rocblas_gemm_strided_batched_ex(
    rocblas_handle handle, rocblas_operation transA, rocblas_operation transB, rocblas_int m,
    rocblas_int n, rocblas_int k, const void* alpha, const void* a, rocblas_datatype a_type,
    rocblas_int lda, int64_t strideA, const void* b, rocblas_datatype b_type, rocblas_int ldb,
    int64_t strideB, const void* beta, const void* c, rocblas_datatype c_type, rocblas_int ldc,
    int64_t strideC, void* d, rocblas_datatype d_type, rocblas_int ldd, int64_t strideD,
    rocblas_int batch_count, rocblas_datatype compute_type, rocblas_gemm_algo algo,
    int32_t solution_index, uint32_t flags);

/* rocBLAS handle calls.  The reference forwarded these untouched (they are
 * not in its export list) and read the stream and pointer mode of its global
 * hipBLAS state.  Without a real rocBLAS on a CUDA machine, rocblas handles
 * are this library's own objects and these calls manage them; with a real
 * rocBLAS loaded, each call is forwarded as well. */
rocblas_status rocblas_create_handle(rocblas_handle* handle);
rocblas_status rocblas_destroy_handle(rocblas_handle handle);
rocblas_status rocblas_set_stream(rocblas_handle handle, hipStream_t stream);
rocblas_status rocblas_get_stream(rocblas_handle handle, hipStream_t* stream);
rocblas_status rocblas_set_pointer_mode(rocblas_handle handle, rocblas_pointer_mode mode);
rocblas_status rocblas_get_pointer_mode(rocblas_handle handle, rocblas_pointer_mode* mode);

#ifdef __cplusplus
}
#endif
