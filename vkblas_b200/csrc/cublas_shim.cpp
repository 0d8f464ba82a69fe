// cublas_shim.cpp -- cuBLAS GEMM interposer over the B200 BLAS core.
//
// Built into its own library, libvkblas_cublas.so, for LD_PRELOAD into a CUDA
// application (PyTorch's `a @ b`, `bmm`).  The hipBLAS shim of the reference
// (lakitu12/vkblas src/vkblas_hipblas.c) reaches no caller on a CUDA machine;
// this is the same idea on the ABI CUDA programs actually bind: the GEMM entry
// points below run on this library's kernels, every other cuBLAS function --
// and every GEMM this library declines -- runs in the real libcublas.
//
// Handles are the real library's (cublasCreate is not intercepted), so their
// stream, pointer mode and math mode are read through the real getters.
// Column-major cuBLAS maps to the engine's row-major contract by swapping the
// operands, as the reference's shim does for hipBLAS (src/vkblas_hipblas.c:
// 234-239).  Declined (forwarded unchanged):
//   - empty problems, k = 0 (C = beta*C), and lda/ldb/ldc the real library
//     rejects -- it returns its own status;
//   - mixed element types, compute types that do not accumulate in fp32,
//     fp16 scalars in device memory (cublasHgemm*);
//   - anything the engine cannot run.
// fp32 GEMMs use the 3xTF32 tensor-core path (fp32-accurate, not bit-equal to
// FFMA) unless the handle's math mode is CUBLAS_PEDANTIC_MATH or the compute
// type is CUBLAS_COMPUTE_32F_PEDANTIC, which select the exact FFMA kernel.
//
// VKBLAS_REAL_CUBLAS names the real library (default libcublas.so.12).
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>

#include <atomic>

#include "vkblas_b200.h"
#include "vkblas_cublas.h"

#define SHIM_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

std::atomic<uint64_t> g_ran{0}, g_forwarded{0};

void* real_cublas() {
    static void* h = [] {
        const char* path = getenv("VKBLAS_REAL_CUBLAS");
        void* r = dlopen(path && *path ? path : "libcublas.so.12", RTLD_LAZY | RTLD_LOCAL);
        if (!r && getenv("VKBLAS_TRACE")) fprintf(stderr, "[vkblas] real cuBLAS not found: %s\n", dlerror());
        return r;
    }();
    return h;
}

template <typename F>
F real_sym(const char* name) {
    void* h = real_cublas();
    return h ? reinterpret_cast<F>(dlsym(h, name)) : nullptr;
}

// Forward to the real function of the same name (NOT_INITIALIZED without it).
#define FORWARD_AS(type, name, ...)                                                \
    ([&]() -> cublasStatus_t {                                                     \
        static auto fn_ = real_sym<type>(#name);                                   \
        g_forwarded.fetch_add(1, std::memory_order_relaxed);                       \
        return fn_ ? fn_(__VA_ARGS__) : CUBLAS_STATUS_NOT_INITIALIZED;             \
    }())
#define FORWARD(name, ...) FORWARD_AS(decltype(&name), name, __VA_ARGS__)

// The C entry points of the two functions cuBLAS's C++ header also overloads.
using GemmEx_fn = cublasStatus_t (*)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int,
                                     int, int, const void*, const void*, cudaDataType_t, int,
                                     const void*, cudaDataType_t, int, const void*, void*,
                                     cudaDataType_t, int, cublasComputeType_t, cublasGemmAlgo_t);
using GemmStridedBatchedEx_fn = cublasStatus_t (*)(
    cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int, const void*, const void*,
    cudaDataType_t, int, long long int, const void*, cudaDataType_t, int, long long int,
    const void*, void*, cudaDataType_t, int, long long int, int, cublasComputeType_t,
    cublasGemmAlgo_t);

struct HandleState {
    cudaStream_t stream;
    cublasPointerMode_t pmode;
    cublasMath_t math;
};

bool handle_state(cublasHandle_t h, HandleState& st) {
    static auto get_stream = real_sym<decltype(&cublasGetStream_v2)>("cublasGetStream_v2");
    static auto get_pmode = real_sym<decltype(&cublasGetPointerMode_v2)>("cublasGetPointerMode_v2");
    static auto get_math = real_sym<decltype(&cublasGetMathMode)>("cublasGetMathMode");
    if (!h || !get_stream || !get_pmode || !get_math) return false;
    return get_stream(h, &st.stream) == CUBLAS_STATUS_SUCCESS &&
           get_pmode(h, &st.pmode) == CUBLAS_STATUS_SUCCESS &&
           get_math(h, &st.math) == CUBLAS_STATUS_SUCCESS;
}

int eng_op(cublasOperation_t op) {
    if (op == CUBLAS_OP_N) return VKBLAS_OP_N;
    if (op == CUBLAS_OP_T || op == CUBLAS_OP_C) return VKBLAS_OP_T;     // real types
    return -1;
}

bool fp32_accumulate(cublasComputeType_t c) {
    return c == CUBLAS_COMPUTE_32F || c == CUBLAS_COMPUTE_32F_PEDANTIC ||
           c == CUBLAS_COMPUTE_32F_FAST_16F || c == CUBLAS_COMPUTE_32F_FAST_16BF ||
           c == CUBLAS_COMPUTE_32F_FAST_TF32 || (int)c == (int)CUDA_R_32F;   // legacy value
}

bool engine_dtype(cudaDataType_t t, vkblas_dtype_t& dt) {
    if (t == CUDA_R_32F) { dt = VKBLAS_DT_F32; return true; }
    if (t == CUDA_R_16F) { dt = VKBLAS_DT_F16; return true; }
    if (t == CUDA_R_16BF) { dt = VKBLAS_DT_BF16; return true; }
    return false;
}

// Run C = alpha op(A) op(B) + beta C (column-major, batched) on this
// library's kernels; false = decline (the caller forwards the call).
bool run(cublasHandle_t handle, vkblas_dtype_t dt, cublasOperation_t ta, cublasOperation_t tb,
         int m, int n, int k, const float* alpha, const void* A, int lda, long long sA,
         const void* B, int ldb, long long sB, const float* beta, void* C, int ldc, long long sC,
         int batch, bool pedantic) {
    if (m <= 0 || n <= 0 || k <= 0 || batch <= 0 || !alpha || !beta || !A || !B || !C) return false;
    const int oa = eng_op(tb), ob = eng_op(ta);
    if (oa < 0 || ob < 0) return false;
    // cuBLAS's own argument rules: leave violations to the real library.
    if (lda < (ta == CUBLAS_OP_N ? m : k) || ldb < (tb == CUBLAS_OP_N ? k : n) || ldc < m) return false;
    if (batch > 1 && (sA < 0 || sB < 0 || sC < 0)) return false;
    HandleState st;
    if (!handle_state(handle, st)) return false;
    // The math mode may carry CUBLAS_MATH_DISALLOW_REDUCED_PRECISION_REDUCTION (a flag).
    const int math = (int)st.math & ~(int)CUBLAS_MATH_DISALLOW_REDUCED_PRECISION_REDUCTION;
    const bool exact = dt == VKBLAS_DT_F32 && (pedantic || math == (int)CUBLAS_PEDANTIC_MATH);
    const int saved = vkblas_b200_get_path();
    if (exact) vkblas_b200_set_path(VKBLAS_PATH_SIMT);
    // Column-major -> row-major: op_a <- transB, op_b <- transA, M <- n, N <- m.
    const vkblas_status_t rc = vkblas_gemm_ex(
        dt, (vkblas_op_t)oa, (vkblas_op_t)ob, (uint32_t)n, (uint32_t)m, (uint32_t)k, alpha, beta,
        st.pmode == CUBLAS_POINTER_MODE_DEVICE, B, (uint32_t)ldb, A, (uint32_t)lda, C,
        (uint32_t)ldc, (uint32_t)batch, batch > 1 ? sB : 0, batch > 1 ? sA : 0,
        batch > 1 ? sC : 0, reinterpret_cast<void*>(st.stream));
    if (exact) vkblas_b200_set_path(saved);
    if (rc != VKBLAS_OK) return false;
    g_ran.fetch_add(1, std::memory_order_relaxed);
    return true;
}

// fp16 scalars (cublasHgemm*) given on the host, widened; false when they are
// device pointers (declined).
bool half_scalars(cublasHandle_t handle, const __half* alpha, const __half* beta, float& a,
                  float& b) {
    HandleState st;
    if (!alpha || !beta || !handle_state(handle, st) || st.pmode != CUBLAS_POINTER_MODE_HOST)
        return false;
    a = __half2float(*alpha);
    b = __half2float(*beta);
    return true;
}

}  // namespace

SHIM_EXPORT cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                                          cublasOperation_t transb, int m, int n, int k,
                                          const float* alpha, const float* A, int lda,
                                          const float* B, int ldb, const float* beta, float* C,
                                          int ldc) {
    if (run(handle, VKBLAS_DT_F32, transa, transb, m, n, k, alpha, A, lda, 0, B, ldb, 0, beta, C,
            ldc, 0, 1, false))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD(cublasSgemm_v2, handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C,
                   ldc);
}

SHIM_EXPORT cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle,
                                                     cublasOperation_t transa,
                                                     cublasOperation_t transb, int m, int n, int k,
                                                     const float* alpha, const float* A, int lda,
                                                     long long int strideA, const float* B, int ldb,
                                                     long long int strideB, const float* beta,
                                                     float* C, int ldc, long long int strideC,
                                                     int batchCount) {
    if (run(handle, VKBLAS_DT_F32, transa, transb, m, n, k, alpha, A, lda, strideA, B, ldb, strideB,
            beta, C, ldc, strideC, batchCount, false))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD(cublasSgemmStridedBatched, handle, transa, transb, m, n, k, alpha, A, lda,
                   strideA, B, ldb, strideB, beta, C, ldc, strideC, batchCount);
}

SHIM_EXPORT cublasStatus_t cublasSgemmEx(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const float* alpha, const void* A, cudaDataType_t Atype,
                                         int lda, const void* B, cudaDataType_t Btype, int ldb,
                                         const float* beta, void* C, cudaDataType_t Ctype,
                                         int ldc) {
    vkblas_dtype_t dt;
    if (Atype == Btype && Btype == Ctype && engine_dtype(Atype, dt) &&
        run(handle, dt, transa, transb, m, n, k, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1,
            false))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD(cublasSgemmEx, handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype,
                   ldb, beta, C, Ctype, ldc);
}

SHIM_EXPORT cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa,
                                        cublasOperation_t transb, int m, int n, int k,
                                        const void* alpha, const void* A, cudaDataType_t Atype,
                                        int lda, const void* B, cudaDataType_t Btype, int ldb,
                                        const void* beta, void* C, cudaDataType_t Ctype, int ldc,
                                        cublasComputeType_t computeType, cublasGemmAlgo_t algo) {
    vkblas_dtype_t dt;
    if (Atype == Btype && Btype == Ctype && engine_dtype(Atype, dt) && fp32_accumulate(computeType) &&
        run(handle, dt, transa, transb, m, n, k, static_cast<const float*>(alpha), A, lda, 0, B, ldb,
            0, static_cast<const float*>(beta), C, ldc, 0, 1,
            computeType == CUBLAS_COMPUTE_32F_PEDANTIC))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD_AS(GemmEx_fn, cublasGemmEx, handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype,
                   ldb, beta, C, Ctype, ldc, computeType, algo);
}

SHIM_EXPORT cublasStatus_t cublasGemmStridedBatchedEx(
    cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb, int m, int n, int k,
    const void* alpha, const void* A, cudaDataType_t Atype, int lda, long long int strideA,
    const void* B, cudaDataType_t Btype, int ldb, long long int strideB, const void* beta, void* C,
    cudaDataType_t Ctype, int ldc, long long int strideC, int batchCount,
    cublasComputeType_t computeType, cublasGemmAlgo_t algo) {
    vkblas_dtype_t dt;
    if (Atype == Btype && Btype == Ctype && engine_dtype(Atype, dt) && fp32_accumulate(computeType) &&
        run(handle, dt, transa, transb, m, n, k, static_cast<const float*>(alpha), A, lda, strideA, B,
            ldb, strideB, static_cast<const float*>(beta), C, ldc, strideC, batchCount,
            computeType == CUBLAS_COMPUTE_32F_PEDANTIC))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD_AS(GemmStridedBatchedEx_fn, cublasGemmStridedBatchedEx, handle, transa, transb, m, n, k, alpha, A, Atype, lda,
                   strideA, B, Btype, ldb, strideB, beta, C, Ctype, ldc, strideC, batchCount,
                   computeType, algo);
}

SHIM_EXPORT cublasStatus_t cublasHgemm(cublasHandle_t handle, cublasOperation_t transa,
                                       cublasOperation_t transb, int m, int n, int k,
                                       const __half* alpha, const __half* A, int lda,
                                       const __half* B, int ldb, const __half* beta, __half* C,
                                       int ldc) {
    float a, b;
    if (half_scalars(handle, alpha, beta, a, b) &&
        run(handle, VKBLAS_DT_F16, transa, transb, m, n, k, &a, A, lda, 0, B, ldb, 0, &b, C, ldc, 0,
            1, false))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD(cublasHgemm, handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C,
                   ldc);
}

SHIM_EXPORT cublasStatus_t cublasHgemmStridedBatched(
    cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb, int m, int n, int k,
    const __half* alpha, const __half* A, int lda, long long int strideA, const __half* B, int ldb,
    long long int strideB, const __half* beta, __half* C, int ldc, long long int strideC,
    int batchCount) {
    float a, b;
    if (half_scalars(handle, alpha, beta, a, b) &&
        run(handle, VKBLAS_DT_F16, transa, transb, m, n, k, &a, A, lda, strideA, B, ldb, strideB, &b,
            C, ldc, strideC, batchCount, false))
        return CUBLAS_STATUS_SUCCESS;
    return FORWARD(cublasHgemmStridedBatched, handle, transa, transb, m, n, k, alpha, A, lda,
                   strideA, B, ldb, strideB, beta, C, ldc, strideC, batchCount);
}

// Calls this library ran (which = 0) and calls it forwarded to the real
// library (which = 1), since load.
SHIM_EXPORT uint64_t vkblas_cublas_calls(int which) {
    return which == 0 ? g_ran.load() : g_forwarded.load();
}
