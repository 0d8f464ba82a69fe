// simt_gemm.cu -- exact SIMT GEMM (fp32 FFMA, any op / ld / batch stride).
//
// The arithmetic of the reference's tile shaders (lakitu12/vkblas
// src/shaders/gemm_f32_64x64_tmpl.comp:117-163, and the half variant
// gemm_half_128x128_bankfree_tmpl.comp:203-228): every output owns one fp32
// accumulator, k is visited in increasing order with one fused multiply-add
// per step, then C = alpha*acc + beta*C with separate roundings (C not read
// when beta == 0) and a round-to-nearest-even store for 2-byte outputs.  The
// result is therefore bit-identical to the sequential-fmaf CPU oracle, which is
// what this kernel is for: the exactness reference beside the tensor-core
// paths, and the path for shapes whose alignment rules out TMA.
//
// B200 mapping: 128x128 CTA tile, 256 threads with an 8x8 register tile each,
// BK = 8 with register double buffering; shared-memory tiles are k-major
// (As[k][m], Bs[k][n]) so the inner loop issues two conflict-free 128-bit
// shared loads per operand per k.  op(A)/op(B) and arbitrary leading
// dimensions are absorbed by the global loaders; no transpose pass exists.
#include "common.cuh"

namespace vkb {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256;

struct SimtArgs {
    int op_a, op_b;
    uint32_t M, N, K;
    float alpha, beta;
    const float* d_alpha;
    const float* d_beta;
    const void* A; uint32_t lda;
    const void* B; uint32_t ldb;
    void* C; uint32_t ldc;
    uint32_t batch;
    int64_t sa, sb, sc;
};

template <typename T>
__device__ __forceinline__ void load_a(const T* A, const SimtArgs& a, uint32_t m0, uint32_t k0,
                                       int tid, float (&r)[4]) {
    if (a.op_a == 0) {                  // A[m*lda + k], k contiguous: 2 threads per row
        uint32_t m = m0 + (tid >> 1), kb = k0 + (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t k = kb + i;
            r[i] = (m < a.M && k < a.K) ? Elem<T>::load(A + (size_t)m * a.lda + k) : 0.f;
        }
    } else {                            // A[k*lda + m], m contiguous: 32 threads per k
        uint32_t k = k0 + (tid >> 5), mb = m0 + (tid & 31) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t m = mb + i;
            r[i] = (m < a.M && k < a.K) ? Elem<T>::load(A + (size_t)k * a.lda + m) : 0.f;
        }
    }
}

template <typename T>
__device__ __forceinline__ void load_b(const T* B, const SimtArgs& a, uint32_t n0, uint32_t k0,
                                       int tid, float (&r)[4]) {
    if (a.op_b == 0) {                  // B[k*ldb + n], n contiguous
        uint32_t k = k0 + (tid >> 5), nb = n0 + (tid & 31) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t n = nb + i;
            r[i] = (n < a.N && k < a.K) ? Elem<T>::load(B + (size_t)k * a.ldb + n) : 0.f;
        }
    } else {                            // B[n*ldb + k], k contiguous
        uint32_t n = n0 + (tid >> 1), kb = k0 + (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t k = kb + i;
            r[i] = (n < a.N && k < a.K) ? Elem<T>::load(B + (size_t)n * a.ldb + k) : 0.f;
        }
    }
}

__device__ __forceinline__ void store_a(float (*As)[BM + 4], int op_a, int tid, const float (&r)[4]) {
    if (op_a == 0) {
        int m = tid >> 1, kb = (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) As[kb + i][m] = r[i];
    } else {
        int k = tid >> 5, mb = (tid & 31) * 4;
        *reinterpret_cast<float4*>(&As[k][mb]) = make_float4(r[0], r[1], r[2], r[3]);
    }
}

__device__ __forceinline__ void store_b(float (*Bs)[BN + 4], int op_b, int tid, const float (&r)[4]) {
    if (op_b == 0) {
        int k = tid >> 5, nb = (tid & 31) * 4;
        *reinterpret_cast<float4*>(&Bs[k][nb]) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
        int n = tid >> 1, kb = (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) Bs[kb + i][n] = r[i];
    }
}

template <typename T>
__global__ void __launch_bounds__(THREADS) simt_gemm_kernel(SimtArgs a) {
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Bs[2][BK][BN + 4];

    float alpha = a.alpha, beta = a.beta;
    load_scalars(a.d_alpha, a.d_beta, alpha, beta);

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const uint32_t m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const uint32_t ktiles = (a.K + BK - 1) / BK;

    for (uint32_t b = blockIdx.z; b < a.batch; b += gridDim.z) {
        const T* A = reinterpret_cast<const T*>(a.A) + a.sa * (int64_t)b;
        const T* B = reinterpret_cast<const T*>(a.B) + a.sb * (int64_t)b;
        T* C = reinterpret_cast<T*>(a.C) + a.sc * (int64_t)b;

        float acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

        float ra[4], rb[4];
        load_a<T>(A, a, m0, 0, tid, ra);
        load_b<T>(B, a, n0, 0, tid, rb);
        store_a(As[0], a.op_a, tid, ra);
        store_b(Bs[0], a.op_b, tid, rb);
        __syncthreads();

        for (uint32_t kt = 0; kt < ktiles; kt++) {
            const int cur = kt & 1;
            const bool more = kt + 1 < ktiles;
            if (more) {
                load_a<T>(A, a, m0, (kt + 1) * BK, tid, ra);
                load_b<T>(B, a, n0, (kt + 1) * BK, tid, rb);
            }
            const uint32_t rem = a.K - kt * BK;
            const int kmax = rem < (uint32_t)BK ? (int)rem : BK;
            // Exactly K steps per output, in order: the tail tile stops at K.
#pragma unroll
            for (int kk = 0; kk < BK; kk++) {
                if (kk < kmax) {
                    float av[8], bv[8];
                    float4 t0 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 4]);
                    float4 t1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + ty * 4]);
                    float4 u0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 4]);
                    float4 u1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tx * 4]);
                    av[0] = t0.x; av[1] = t0.y; av[2] = t0.z; av[3] = t0.w;
                    av[4] = t1.x; av[5] = t1.y; av[6] = t1.z; av[7] = t1.w;
                    bv[0] = u0.x; bv[1] = u0.y; bv[2] = u0.z; bv[3] = u0.w;
                    bv[4] = u1.x; bv[5] = u1.y; bv[6] = u1.z; bv[7] = u1.w;
#pragma unroll
                    for (int i = 0; i < 8; i++)
#pragma unroll
                        for (int j = 0; j < 8; j++) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
                }
            }
            if (more) {
                store_a(As[cur ^ 1], a.op_a, tid, ra);
                store_b(Bs[cur ^ 1], a.op_b, tid, rb);
            }
            __syncthreads();
        }

#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
            if (m >= a.M) continue;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
                if (n >= a.N) continue;
                T* cp = C + (size_t)m * a.ldc + n;
                const float c = (beta != 0.f) ? Elem<T>::to_f(*cp) : 0.f;
                *cp = Elem<T>::from_f(epilogue(alpha, acc[i][j], beta, c));
            }
        }
    }
}

}  // namespace

cudaError_t launch_simt_gemm(const GemmProblem& p, cudaStream_t s) {
    SimtArgs a;
    a.op_a = p.op_a; a.op_b = p.op_b;
    a.M = p.M; a.N = p.N; a.K = p.K;
    a.alpha = p.alpha; a.beta = p.beta; a.d_alpha = p.d_alpha; a.d_beta = p.d_beta;
    a.A = p.A; a.lda = p.lda; a.B = p.B; a.ldb = p.ldb; a.C = p.C; a.ldc = p.ldc;
    a.batch = p.batch; a.sa = p.sa; a.sb = p.sb; a.sc = p.sc;
    if ((p.M + BM - 1) / BM > 65535u) return cudaErrorInvalidConfiguration;
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, p.batch < 65535u ? p.batch : 65535u);
    switch (p.dtype) {
        case DT_F32: simt_gemm_kernel<float><<<grid, THREADS, 0, s>>>(a); break;
        case DT_F16: simt_gemm_kernel<__half><<<grid, THREADS, 0, s>>>(a); break;
        case DT_BF16: simt_gemm_kernel<__nv_bfloat16><<<grid, THREADS, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    count_launch();
    return cudaGetLastError();
}

}  // namespace vkb
