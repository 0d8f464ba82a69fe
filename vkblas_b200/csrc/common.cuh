// common.cuh -- shared definitions of the B200 BLAS core kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cuda.h>

namespace vkb {

// Element types of the engine (values match vkblas_dtype_t).
enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

// One GEMM call in the engine's row-major contract (reference
// src/vkblas.h:19-26): C[M,N] = alpha*op(A)*op(B) + beta*C per batch entry.
struct GemmProblem {
    int dtype;
    int op_a, op_b;                 // 0 = N, 1 = T
    uint32_t M, N, K;
    float alpha, beta;              // used when d_alpha / d_beta are null
    const float* d_alpha;           // device-resident scalars (pointer mode DEVICE)
    const float* d_beta;
    const void* A; uint32_t lda;
    const void* B; uint32_t ldb;
    void* C; uint32_t ldc;
    uint32_t batch;
    int64_t sa, sb, sc;             // element strides between batch entries (0 = broadcast)
};

// Device status codes written by bounded waits that ran out.
enum DeviceStatus : int {
    DS_OK = 0,
    DS_TIMEOUT_PRODUCER = 1,
    DS_TIMEOUT_MMA = 2,
    DS_TIMEOUT_EPILOGUE = 3,
    DS_TIMEOUT_TRANSFORM = 4,
};

// Element load/store through fp32.
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float load(const float* p) { return *p; }
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// The reference epilogue `alpha*acc + beta*c` (gemm_f32_64x64_tmpl.comp:158-160)
// with both products and the sum rounded separately (no contraction), and c
// not read when beta == 0.
__device__ __forceinline__ float epilogue(float alpha, float acc, float beta, float c) {
    return __fadd_rn(__fmul_rn(alpha, acc), __fmul_rn(beta, c));
}

__device__ __forceinline__ void load_scalars(const float* d_alpha, const float* d_beta,
                                             float& alpha, float& beta) {
    if (d_alpha) alpha = *d_alpha;
    if (d_beta) beta = *d_beta;
}

}  // namespace vkb

// Kernel launchers (host side), one per translation unit.
namespace vkb {
cudaError_t launch_simt_gemm(const GemmProblem& p, cudaStream_t s);
bool gemv_supported(const GemmProblem& p);
int gemv_auto_splitk(const GemmProblem& p, int num_sms);
size_t gemv_workspace_bytes(const GemmProblem& p, int splitk);
cudaError_t launch_gemv(const GemmProblem& p, int splitk, void* workspace, int* d_status,
                        cudaStream_t s);
bool gemv_f32_supported(const GemmProblem& p);
int gemv_f32_auto_splitk(const GemmProblem& p, int num_sms);
size_t gemv_f32_workspace_bytes(const GemmProblem& p, int splitk);
cudaError_t launch_gemv_f32(const GemmProblem& p, int splitk, void* workspace, cudaStream_t s);
bool umma_supported(const GemmProblem& p);
bool umma_profitable(const GemmProblem& p);
size_t umma_workspace_bytes(const GemmProblem& p);
// Split-K / wave-tail scratch: fp32 partial tiles of the split units; 0 = no split.
size_t umma_split_workspace_bytes(const GemmProblem& p, int num_sms);
int umma_split_count(const GemmProblem& p, int num_sms);   // K splits of the last wave (1 = none)
// True when the call runs on 2-CTA clusters (256-row tiles, cta_group::2).
bool umma_uses_pair(const GemmProblem& p, int num_sms, bool split_ws);
int umma_tile_n(const GemmProblem& p);                      // N width of the kernel's tile
// Tile and split plan of a tensor-core GEMM (pure host logic, see
// vkblas_b200_tc_plan); allow_wide: 256-wide 3xTF32 pair tiles may be chosen.
struct UmmaPlan {
    uint32_t tile_m, tile_n, transposed, pair;
    uint32_t tiles, full_tiles, splits, kblocks, kblocks_per_split;
    uint64_t partial_bytes;
    uint32_t tail_tiles;     // last-wave tiles run as two 256 x 128 halves each
    bool too_many_tiles;     // 2^31 tiles or more: the launch path rejects the call
};
UmmaPlan umma_plan(const GemmProblem& p, int num_sms, bool allow_wide);
// cudaErrorNotSupported: the operands cannot be described to TMA (nothing launched).
// test_stall: test hook, the producer leaves the first stage empty so the
// MMA warp's bounded wait runs out (status DS_TIMEOUT_MMA) after 20 ms.
// ev_start / ev_end (may be null): recorded on `s` right before the GEMM
// kernel (after any 3xTF32 pre-pass) and right after it (after the split
// reduce, if any) -- the measurement hook vkblas_b200_set_kernel_events.
// peers / npeers (<= 7): pointers, valid in this process, to other copies of
// C with C's layout; every element the kernels write to C is written to each
// of them too (cudaErrorInvalidValue for more than 7 or a null pointer,
// cudaErrorNotSupported for a small-M transposed problem).
cudaError_t launch_umma_gemm(const GemmProblem& p, int num_sms, int* d_status, void* workspace,
                             void* split_workspace, bool test_stall, cudaStream_t s,
                             cudaEvent_t ev_start = nullptr, cudaEvent_t ev_end = nullptr,
                             void* const* peers = nullptr, uint32_t npeers = 0);
// 2-D TMA tensor map over a 2-byte matrix [outer][inner] (row stride ld
// elements), box [box_outer][box_inner], no swizzle.  False if the driver
// entry point is missing or the layout cannot be described.
bool encode_tmap_2d(CUtensorMap* m, bool bf16, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t ld, uint32_t box_inner, uint32_t box_outer);
// fp64 GEMM (exact sequential fma) and the complex planar helpers (dgemm.cu).
cudaError_t launch_dgemm(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K, double alpha,
                         const double* A, uint32_t lda, const double* B, uint32_t ldb, double beta,
                         double* C, uint32_t ldc, uint32_t batch, int64_t sa, int64_t sb,
                         int64_t sc, cudaStream_t s);
cudaError_t launch_cx_split(bool dbl, const void* src, uint32_t rows, uint32_t cols, uint32_t ld,
                            int64_t stride, uint32_t batch, void* re, void* im, cudaStream_t s);
cudaError_t launch_cx_combine(bool dbl, const void* t1, const void* t2, void* C, uint32_t M,
                              uint32_t N, uint32_t ldc, int64_t sc, uint32_t batch, double ar,
                              double ai, double br, double bi, cudaStream_t s);
// Host-side launch counter (all kernels of this library).
void count_launch();
}  // namespace vkb
