/* Minimal stand-in for <hipblas/hipblas.h>, used ONLY to compile the
 * reference's own CPU GEMM checkers (test/test_gemm.c, test/test_h.c) into
 * oracle/_ref/ on a machine without ROCm.  The checkers use nothing from
 * hipBLAS except these names; the device-side calls in their main() are never
 * executed (main is renamed away by the wrapper translation units).
 * Enum values follow the public hipBLAS header (HIPBLAS_OP_N=111,
 * HIPBLAS_OP_T=112, HIPBLAS_STATUS_SUCCESS=0). */
#pragma once
#include "../hip/hip_runtime_api.h"

typedef void* hipblasHandle_t;
typedef enum { HIPBLAS_OP_N = 111, HIPBLAS_OP_T = 112, HIPBLAS_OP_C = 113 } hipblasOperation_t;
typedef enum { HIPBLAS_STATUS_SUCCESS = 0, HIPBLAS_STATUS_NOT_SUPPORTED = 7 } hipblasStatus_t;
typedef int hipblasDatatype_t;
typedef int hipblasComputeType_t;
typedef int hipblasGemmAlgo_t;
#define HIPBLAS_R_16F 150
#define HIPBLAS_R_32F 151
#define HIPBLAS_R_16B 168
#define HIPBLAS_COMPUTE_32F 2
#define HIPBLAS_GEMM_DEFAULT 100
