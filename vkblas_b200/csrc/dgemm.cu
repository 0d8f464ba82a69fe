// dgemm.cu -- fp64 GEMM and the complex64 / complex128 helpers.
//
// Replaces the reference's fp64 and complex fallbacks (lakitu12/vkblas
// src/vkblas.c:3653-4188, shaders gemm_f64_32x32_tmpl.comp, cvt_cx.comp,
// cvt_cz.comp, cx_combine.comp, cx_combine_d64.comp):
//   - fp64 GEMM: every output owns one double accumulator, k in increasing
//     order with one fused multiply-add per step (gemm_f64_32x32_tmpl.comp:
//     85-100), then C = alpha*acc + beta*C with separate roundings, C not read
//     when beta == 0 (:116-117).  Bit-identical to the sequential fma oracle.
//   - complex GEMMs run as four real GEMMs on planar copies (the engine's
//     fp32 GEMM for complex64, the kernel below for complex128):
//       T1 = Ar*Br;  T1 = -1*(Ai*Bi) + 1*T1;  T2 = Ar*Bi;  T2 = 1*(Ai*Br) + 1*T2
//     (vkblas.c:3816-3823), then the combine
//       C.r = ar*T1 - ai*T2 + br*C.r - bi*C.i,  C.i = ar*T2 + ai*T1 + br*C.i + bi*C.r
//     left to right with separate roundings, the beta terms only when beta is
//     non-zero (cx_combine.comp:32-45).
// Planar copies keep the interleaved operand's element offsets (ld and batch
// stride), so the real GEMMs read them with the caller's leading dimensions.
#include "common.cuh"

namespace vkb {
namespace {

// 64 x 128 CTA tile, 128 threads, 8 x 8 outputs per thread: rows ty*2 + i +
// 16*g (i < 2, g < 4), columns tx*2 + j + 32*h (j < 2, h < 4).  A k step reads
// eight 128-bit fragments (two doubles each) from k-major shared tiles for 64
// FMAs, half the shared-memory traffic per FMA of a 4 x 4 tile.  Fragment
// reads are conflict-free: 16 lanes
// cover 256 contiguous bytes of a B row, and the A reads of a warp are two
// broadcasts.  Global k-tiles arrive by cp.async into two shared stages (no
// registers held), so tile k + 1 lands while tile k is multiplied.
constexpr int DBM = 64, DBN = 128, DBK = 8, DTHREADS = 128;

struct DArgs {
    int op_a, op_b;
    uint32_t M, N, K;
    double alpha, beta;
    const double* A; uint32_t lda;
    const double* B; uint32_t ldb;
    double* C; uint32_t ldc;
    int64_t sa, sb, sc;
    uint32_t batch;
};

// 8-byte asynchronous copy global -> shared; `valid` false writes zero and
// reads nothing.
__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(d), "l"(src),
                 "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One k-tile of an operand (R rows/columns x 8 k) -> shared memory S[k][r],
// R * 8 / 128 elements per thread, in an order that keeps global loads
// coalesced: along k for a k-contiguous operand, along r otherwise.
template <int R>
__device__ __forceinline__ void load_dtile(const double* X, bool k_contig, uint32_t ld,
                                           uint32_t rows, uint32_t K, uint32_t r0, uint32_t k0,
                                           int tid, double (*S)[R + 2]) {
    constexpr int PER = R * DBK / DTHREADS;
#pragma unroll
    for (int q = 0; q < PER; q++) {
        const int e = q * DTHREADS + tid;
        int r, k;
        if (k_contig) { r = e >> 3; k = e & 7; }      // X[r*ld + k]
        else { k = e / R; r = e % R; }                // X[k*ld + r]
        const uint32_t gr = r0 + r, gk = k0 + k;
        const bool in = gr < rows && gk < K;
        const double* src = in ? (k_contig ? X + (size_t)gr * ld + gk : X + (size_t)gk * ld + gr) : X;
        cp_async8(&S[k][r], src, in);
    }
}

__global__ void __launch_bounds__(DTHREADS) dgemm_kernel(DArgs a) {
    __shared__ __align__(16) double As[2][DBK][DBM + 2];  // [stage][k][m]
    __shared__ __align__(16) double Bs[2][DBK][DBN + 2];  // [stage][k][n]
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const uint32_t m0 = blockIdx.y * DBM, n0 = blockIdx.x * DBN;
    const bool a_kc = a.op_a == 0, b_kc = a.op_b != 0;
    for (uint32_t b = blockIdx.z; b < a.batch; b += gridDim.z) {
    const double* A = a.A + a.sa * (int64_t)b;
    const double* B = a.B + a.sb * (int64_t)b;
    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0;
    const uint32_t ktiles = (a.K + DBK - 1) / DBK;
    load_dtile<DBM>(A, a_kc, a.lda, a.M, a.K, m0, 0, tid, As[0]);
    load_dtile<DBN>(B, b_kc, a.ldb, a.N, a.K, n0, 0, tid, Bs[0]);
    cp_async_commit();
    for (uint32_t kt = 0; kt < ktiles; kt++) {
        const uint32_t k0 = kt * DBK;
        const int st = kt & 1;
        if (kt + 1 < ktiles) {             // next tile into the other stage
            load_dtile<DBM>(A, a_kc, a.lda, a.M, a.K, m0, k0 + DBK, tid, As[st ^ 1]);
            load_dtile<DBN>(B, b_kc, a.ldb, a.N, a.K, n0, k0 + DBK, tid, Bs[st ^ 1]);
            cp_async_commit();
            cp_async_wait<1>();            // this tile's group has landed
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t kend = min((uint32_t)DBK, a.K - k0);   // stop at K: no extra terms
#pragma unroll
        for (int kk = 0; kk < DBK; kk++) {
            if ((uint32_t)kk < kend) {
                double2 fa[4], fb[4];
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    fa[g] = *reinterpret_cast<const double2*>(&As[st][kk][ty * 2 + 16 * g]);
                    fb[g] = *reinterpret_cast<const double2*>(&Bs[st][kk][tx * 2 + 32 * g]);
                }
#pragma unroll
                for (int g = 0; g < 4; g++)
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        acc[2 * g][2 * h] = __fma_rn(fa[g].x, fb[h].x, acc[2 * g][2 * h]);
                        acc[2 * g][2 * h + 1] = __fma_rn(fa[g].x, fb[h].y, acc[2 * g][2 * h + 1]);
                        acc[2 * g + 1][2 * h] = __fma_rn(fa[g].y, fb[h].x, acc[2 * g + 1][2 * h]);
                        acc[2 * g + 1][2 * h + 1] = __fma_rn(fa[g].y, fb[h].y, acc[2 * g + 1][2 * h + 1]);
                    }
            }
        }
        __syncthreads();                   // stage st is refilled two tiles on
    }
    double* C = a.C + a.sc * (int64_t)b;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t m = m0 + ty * 2 + (i & 1) + 16 * (i >> 1);
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t n = n0 + tx * 2 + (j & 1) + 32 * (j >> 1);
            if (n >= a.N) continue;
            double* c = C + (size_t)m * a.ldc + n;
            const double old = (a.beta != 0.0) ? *c : 0.0;
            *c = __dadd_rn(__dmul_rn(a.alpha, acc[i][j]), __dmul_rn(a.beta, old));
        }
    }
    }   // batch entries, striding by gridDim.z
}

// Interleaved complex [b*stride + r*ld + c] -> real and imaginary planes at
// the same element offsets, for r < rows, c < cols.
template <typename T>
__global__ void cx_split_kernel(const T* __restrict__ src, uint32_t rows, uint32_t cols,
                                uint32_t ld, int64_t stride, uint32_t batch, T* __restrict__ re,
                                T* __restrict__ im) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    for (uint32_t b = blockIdx.z; b < batch; b += gridDim.z)
        for (uint32_t r = blockIdx.y; r < rows; r += gridDim.y) {
            const size_t o = (size_t)(stride * (int64_t)b) + (size_t)r * ld + c;
            re[o] = src[2 * o];
            im[o] = src[2 * o + 1];
        }
}

__device__ __forceinline__ float mul_rn(float x, float y) { return __fmul_rn(x, y); }
__device__ __forceinline__ double mul_rn(double x, double y) { return __dmul_rn(x, y); }
__device__ __forceinline__ float add_rn(float x, float y) { return __fadd_rn(x, y); }
__device__ __forceinline__ double add_rn(double x, double y) { return __dadd_rn(x, y); }
__device__ __forceinline__ float sub_rn(float x, float y) { return __fsub_rn(x, y); }
__device__ __forceinline__ double sub_rn(double x, double y) { return __dsub_rn(x, y); }

// C = alpha * (T1 + i T2) + beta * C over M x N per batch entry (C interleaved).
template <typename T>
__global__ void cx_combine_kernel(const T* __restrict__ t1, const T* __restrict__ t2, T* C,
                                  uint32_t M, uint32_t N, uint32_t ldc, int64_t sc, uint32_t batch,
                                  T ar, T ai, T br, T bi) {
    const uint32_t n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    for (uint32_t b = blockIdx.z; b < batch; b += gridDim.z)
    for (uint32_t m = blockIdx.y; m < M; m += gridDim.y) {
        const size_t o = (size_t)(sc * (int64_t)b) + (size_t)m * ldc + n;
        const T fr = t1[o], fi = t2[o];
        T outr = sub_rn(mul_rn(ar, fr), mul_rn(ai, fi));
        T outi = add_rn(mul_rn(ar, fi), mul_rn(ai, fr));
        if (br != T(0) || bi != T(0)) {
            const T r0 = C[2 * o], i0 = C[2 * o + 1];
            outr = sub_rn(add_rn(outr, mul_rn(br, r0)), mul_rn(bi, i0));
            outi = add_rn(add_rn(outi, mul_rn(br, i0)), mul_rn(bi, r0));
        }
        C[2 * o] = outr;
        C[2 * o + 1] = outi;
    }
}

}  // namespace

cudaError_t launch_dgemm(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K, double alpha,
                         const double* A, uint32_t lda, const double* B, uint32_t ldb, double beta,
                         double* C, uint32_t ldc, uint32_t batch, int64_t sa, int64_t sb,
                         int64_t sc, cudaStream_t s) {
    DArgs a{op_a, op_b, M, N, K, alpha, beta, A, lda, B, ldb, C, ldc, sa, sb, sc, batch};
    const dim3 grid((N + DBN - 1) / DBN, (M + DBM - 1) / DBM, batch < 65535u ? batch : 65535u);
    if (grid.y > 65535) return cudaErrorInvalidConfiguration;
    dgemm_kernel<<<grid, DTHREADS, 0, s>>>(a);
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_cx_split(bool dbl, const void* src, uint32_t rows, uint32_t cols, uint32_t ld,
                            int64_t stride, uint32_t batch, void* re, void* im, cudaStream_t s) {
    const uint32_t nb = stride ? batch : 1u;        // a broadcast operand is split once
    const dim3 grid((cols + 255) / 256, rows < 65535u ? rows : 65535u, nb < 65535u ? nb : 65535u);
    if (dbl)
        cx_split_kernel<double><<<grid, 256, 0, s>>>(static_cast<const double*>(src), rows, cols,
                                                       ld, stride, nb, static_cast<double*>(re),
                                                       static_cast<double*>(im));
    else
        cx_split_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(src), rows, cols, ld,
                                                      stride, nb, static_cast<float*>(re),
                                                      static_cast<float*>(im));
    count_launch();
    return cudaGetLastError();
}

cudaError_t launch_cx_combine(bool dbl, const void* t1, const void* t2, void* C, uint32_t M,
                              uint32_t N, uint32_t ldc, int64_t sc, uint32_t batch, double ar,
                              double ai, double br, double bi, cudaStream_t s) {
    const dim3 grid((N + 255) / 256, M < 65535u ? M : 65535u, batch < 65535u ? batch : 65535u);
    if (dbl)
        cx_combine_kernel<double><<<grid, 256, 0, s>>>(
            static_cast<const double*>(t1), static_cast<const double*>(t2), static_cast<double*>(C),
            M, N, ldc, sc, batch, ar, ai, br, bi);
    else
        cx_combine_kernel<float><<<grid, 256, 0, s>>>(
            static_cast<const float*>(t1), static_cast<const float*>(t2), static_cast<float*>(C), M,
            N, ldc, sc, batch, (float)ar, (float)ai, (float)br, (float)bi);
    count_launch();
    return cudaGetLastError();
}

}  // namespace vkb
