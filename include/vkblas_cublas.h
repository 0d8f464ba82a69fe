/* vkblas_cublas.h -- the cuBLAS GEMM interposer, libvkblas_cublas.so.
 *
 * No counterpart in the reference: its shim (src/vkblas_hipblas.c) serves the
 * hipBLAS ABI, which CUDA programs do not call.  This library serves the same
 * purpose on CUDA: loaded with LD_PRELOAD into an application that links the
 * real libcublas.so.12, it defines these cuBLAS entry points (signatures and
 * enum values from cuBLAS's public cublas_v2.h, exported under the symbol
 * version libcublas.so.12 that applications bind):
 *
 *   cublasSgemm_v2, cublasSgemmStridedBatched, cublasSgemmEx, cublasGemmEx,
 *   cublasGemmStridedBatchedEx, cublasHgemm, cublasHgemmStridedBatched
 *
 * Each runs on this library's kernels when it can (same element type for A,
 * B and C among fp32/fp16/bf16, fp32 accumulation, valid leading dimensions,
 * m, n, k, batch > 0) on the handle's stream, honouring the handle's pointer
 * mode; otherwise it calls the real function unchanged.  Every other cuBLAS
 * function is the real library's.  fp32 runs as 3xTF32 unless the handle's
 * math mode is CUBLAS_PEDANTIC_MATH or the compute type
 * CUBLAS_COMPUTE_32F_PEDANTIC (then the exact FFMA kernel).
 * VKBLAS_REAL_CUBLAS overrides the real library's path.
 */
#ifndef VKBLAS_CUBLAS_H
#define VKBLAS_CUBLAS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Calls this library ran on its own kernels (which = 0) and calls it passed
 * to the real library (which = 1) since it was loaded. */
uint64_t vkblas_cublas_calls(int which);

#ifdef __cplusplus
}
#endif

#endif
