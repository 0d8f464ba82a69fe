/* vkblas.h -- B200-native BLAS core, C API.
 *
 * Drop-in for the engine API of lakitu12/vkblas (src/vkblas.h:1-118): the
 * same status and op enums with the same values, the same function names and
 * the same argument meaning.  Each entry point cites the reference
 * declaration it replaces.
 *
 * Contract (reference src/vkblas.h:19-26), row-major:
 *     C[M,N] = alpha * op(A)[M,K] @ op(B)[K,N] + beta * C
 *     op_a == VKBLAS_OP_T reads A[k*lda + m], else A[m*lda + k]; B likewise
 *     (op_b == VKBLAS_OP_T reads B[n*ldb + k], else B[k*ldb + n]).
 *     Leading dimensions and batch strides are in elements; a batch stride of
 *     0 broadcasts that operand.  beta == 0 means C is not read.
 *
 * Differences that come from the hardware, not from the contract:
 *   - Pointers are CUDA device pointers (or any pointer the current CUDA
 *     device can dereference), used directly; there is no import step.
 *   - Work is enqueued on the calling thread's vkblas stream (see
 *     vkblas_b200.h: vkblas_set_stream; default is the legacy default
 *     stream, so a following blocking cudaMemcpy sees the result).  The
 *     reference returned only after the GPU finished (vkQueueWaitIdle).
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference src/vkblas.h:6-12 (values identical) */
typedef enum {
    VKBLAS_OK = 0,
    VKBLAS_ERR_INIT,      /* no usable CUDA device / kernel image            */
    VKBLAS_ERR_IMPORT,    /* kept for ABI parity; not produced on CUDA        */
    VKBLAS_ERR_PARAM,     /* invalid argument (zero size, null pointer, ...)  */
    VKBLAS_ERR_FALLBACK   /* operation not handled here: caller should fall back */
} vkblas_status_t;

/* reference src/vkblas.h:14 */
typedef enum { VKBLAS_OP_N = 0, VKBLAS_OP_T = 1 } vkblas_op_t;

/* reference src/vkblas.h:16-19.  The reference invalidates its dma-buf
 * import cache here.  CUDA pointers are used directly, so there is nothing
 * to invalidate: a no-op kept so existing callers link. */
void vkblas_cache_invalidate_base(const void* ptr);

/* reference src/vkblas.h:28-36 (vkblas.c:3104).  fp32 GEMM.
 * Default kernel: 3xTF32 split-precision tcgen05 GEMM when the operands meet
 * its alignment rules, else the exact FFMA SIMT GEMM (sequential fp32
 * accumulation per output, the reference shader's arithmetic). */
vkblas_status_t vkblas_gemm_f32(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    float alpha,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    float beta,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

/* reference src/vkblas.h:41-49 (vkblas.c:3485).  bf16 in/out, fp32
 * accumulate, RNE store.  Same kernels as the fp16 path with bf16 operands. */
vkblas_status_t vkblas_gemm_bf16(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    float alpha,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    float beta,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

/* reference src/vkblas.h:54-62 (vkblas.c:3500).  The reference needed a
 * separate entry to skip a transpose when B arrives in hipBLAS's physical
 * layout.  Operand layouts are absorbed by the kernels' tile loaders here, so
 * this has exactly the semantics of vkblas_gemm_bf16. */
vkblas_status_t vkblas_gemm_bf16_hipblas(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    float alpha,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    float beta,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

/* reference src/vkblas.h:66-74 (vkblas.c:3517).  fp16 in/out, fp32
 * accumulate, RNE store.  Decode shapes (M <= 16, op_b == T) take the split-K
 * GEMV kernel; larger shapes the tcgen05 HGEMM; shapes whose alignment rules
 * out TMA take the exact SIMT kernel. */
vkblas_status_t vkblas_gemm_f16(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    float alpha,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    float beta,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

/* reference src/vkblas.h:79-88, 92-100, 105-114.  Same row-major contract
 * as the others, on the thread's vkblas stream; A, B and C are complex
 * interleaved (8- or 16-byte elements) or double, ld and strides in
 * elements, alpha / beta by value.  fp64 runs an exact fp64 GEMM (one fma per
 * k in order, then alpha*acc + beta*C); complex64 / complex128 run four real
 * GEMMs on planar copies plus a combine, as the reference does
 * (src/vkblas.c:3748-3930).  Returns 0 when done, non-zero when not run
 * (invalid arguments, no usable GPU): the caller then forwards to a real
 * library, as the reference defines. */
int vkblas_gemm_c64(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    float alpha_r, float alpha_i,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    float beta_r, float beta_i,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

int vkblas_gemm_f64(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    double alpha,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    double beta,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

int vkblas_gemm_z64(
    vkblas_op_t op_a, vkblas_op_t op_b,
    uint32_t M, uint32_t N, uint32_t K,
    double alpha_r, double alpha_i,
    const void* A, uint32_t lda,
    const void* B, uint32_t ldb,
    double beta_r, double beta_i,
    void* C, uint32_t ldc,
    uint32_t batch,
    int64_t stride_a, int64_t stride_b, int64_t stride_c);

#ifdef __cplusplus
}
#endif
