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
// B200 mapping: 128x128 CTA tile, 128 threads with a 16x8 register tile each
// (rows ty*4 + i + 32*g, columns tx*4 + j + 64*h), BK = 8.  Shared-memory
// tiles are k-major (As[k][m], Bs[k][n]); a k step reads six conflict-free
// 128-bit fragments for 128 FMAs, and the fragments of step k + 1 are read
// while step k's FMAs issue.  Shared-memory bandwidth is what bounds a SIMT
// GEMM here: an 8x8 tile per thread (four fragments for 64 FMAs) kept the
// L1/shared pipe at 75% with the FMA pipe at 52%.  op(A)/op(B) and arbitrary
// leading dimensions are absorbed by the global loaders; no transpose pass
// exists.
#include "common.cuh"

namespace vkb {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 128;

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
    uint32_t vec_a, vec_b;      // 4-element groups of the operand are vector-aligned
};

// Four consecutive elements as floats, one 128-bit (fp32) or 64-bit (2-byte
// types) load.
template <typename T> __device__ __forceinline__ void load4(const T* p, float* v);
template <> __device__ __forceinline__ void load4<float>(const float* p, float* v) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
template <> __device__ __forceinline__ void load4<__half>(const __half* p, float* v) {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
template <> __device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// One k-tile of an operand (128 rows/columns x 8 k) -> 8 registers per thread,
// as two groups of 4 consecutive elements in memory:
//   k contiguous (A with op_a == 0, B with op_b == 1): rows tid/2 and
//     64 + tid/2, k (tid % 2) * 4 .. +3 -- a warp load covers 16 rows x 32 B;
//   m (or n) contiguous: k = tid / 16, elements (tid % 16) * 4 .. +3 and
//     64 + the same -- a warp load covers 2 k-rows x 256 B, and the shared-
//     memory stores are two conflict-free 128-bit stores.
// `vec`: the operand's base, leading dimension and batch stride keep every
// group vector-aligned; groups that cross the matrix edge load element-wise.
template <typename T>
__device__ __forceinline__ void load_tile(const T* X, bool k_contig, bool vec, uint32_t ld,
                                          uint32_t rows, uint32_t K, uint32_t r0, uint32_t k0,
                                          int tid, float (&r)[8]) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
        uint32_t row, k;
        if (k_contig) {
            row = r0 + (tid >> 1) + 64 * q;
            k = k0 + (tid & 1) * 4;
        } else {
            row = r0 + (tid & 15) * 4 + 64 * q;
            k = k0 + (tid >> 4);
        }
        float* v = r + 4 * q;
        const T* p = k_contig ? X + (size_t)row * ld + k : X + (size_t)k * ld + row;
        const bool whole = k_contig ? (row < rows && k + 3 < K) : (row + 3 < rows && k < K);
        if (vec && whole) {
            load4<T>(p, v);
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const bool in = k_contig ? (row < rows && k + i < K) : (row + i < rows && k < K);
                v[i] = in ? Elem<T>::load(p + i) : 0.f;
            }
        }
    }
}

__device__ __forceinline__ void store_tile(float (*S)[BM + 4], bool k_contig, int tid,
                                           const float (&r)[8]) {
    if (k_contig) {
        const int m = tid >> 1, kb = (tid & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            S[kb + i][m] = r[i];
            S[kb + i][64 + m] = r[4 + i];
        }
    } else {
        const int k = tid >> 4, c = (tid & 15) * 4;
        *reinterpret_cast<float4*>(&S[k][c]) = make_float4(r[0], r[1], r[2], r[3]);
        *reinterpret_cast<float4*>(&S[k][64 + c]) = make_float4(r[4], r[5], r[6], r[7]);
    }
}

// acc[g*4 + i][h*4 + j] += A(row ty*4 + i + 32g) * B(column tx*4 + j + 64h).
__device__ __forceinline__ void fma_step(float (&acc)[16][8], const float4 (&fa)[4],
                                         const float4 (&fb)[2]) {
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const float av[4] = {fa[g].x, fa[g].y, fa[g].z, fa[g].w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float* c = acc[g * 4 + i] + h * 4;
                c[0] = __fmaf_rn(av[i], fb[h].x, c[0]);
                c[1] = __fmaf_rn(av[i], fb[h].y, c[1]);
                c[2] = __fmaf_rn(av[i], fb[h].z, c[2]);
                c[3] = __fmaf_rn(av[i], fb[h].w, c[3]);
            }
        }
    }
}

__device__ __forceinline__ void load_frags(const float (*As)[BM + 4], const float (*Bs)[BN + 4],
                                           int kk, int ty, int tx, float4 (&fa)[4],
                                           float4 (&fb)[2]) {
#pragma unroll
    for (int g = 0; g < 4; g++) fa[g] = *reinterpret_cast<const float4*>(&As[kk][ty * 4 + 32 * g]);
#pragma unroll
    for (int h = 0; h < 2; h++) fb[h] = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4 + 64 * h]);
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
    const bool a_kc = a.op_a == 0, b_kc = a.op_b != 0;

    for (uint32_t b = blockIdx.z; b < a.batch; b += gridDim.z) {
        const T* A = reinterpret_cast<const T*>(a.A) + a.sa * (int64_t)b;
        const T* B = reinterpret_cast<const T*>(a.B) + a.sb * (int64_t)b;
        T* C = reinterpret_cast<T*>(a.C) + a.sc * (int64_t)b;

        float acc[16][8];
#pragma unroll
        for (int i = 0; i < 16; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

        float ra[8], rb[8];
        load_tile<T>(A, a_kc, a.vec_a != 0, a.lda, a.M, a.K, m0, 0, tid, ra);
        load_tile<T>(B, b_kc, a.vec_b != 0, a.ldb, a.N, a.K, n0, 0, tid, rb);
        store_tile(As[0], a_kc, tid, ra);
        store_tile(Bs[0], b_kc, tid, rb);
        __syncthreads();

        for (uint32_t kt = 0; kt < ktiles; kt++) {
            const int cur = kt & 1;
            const bool more = kt + 1 < ktiles;
            if (more) {
                load_tile<T>(A, a_kc, a.vec_a != 0, a.lda, a.M, a.K, m0, (kt + 1) * BK, tid, ra);
                load_tile<T>(B, b_kc, a.vec_b != 0, a.ldb, a.N, a.K, n0, (kt + 1) * BK, tid, rb);
            }
            const uint32_t rem = a.K - kt * BK;
            if (rem >= (uint32_t)BK) {
                float4 fa[2][4], fb[2][2];
                load_frags(As[cur], Bs[cur], 0, ty, tx, fa[0], fb[0]);
#pragma unroll
                for (int kk = 0; kk < BK; kk++) {
                    if (kk + 1 < BK) load_frags(As[cur], Bs[cur], kk + 1, ty, tx, fa[(kk + 1) & 1], fb[(kk + 1) & 1]);
                    fma_step(acc, fa[kk & 1], fb[kk & 1]);
                }
            } else {
                // Exactly K steps per output, in order: the tail tile stops at K.
                for (uint32_t kk = 0; kk < rem; kk++) {
                    float4 fa[4], fb[2];
                    load_frags(As[cur], Bs[cur], (int)kk, ty, tx, fa, fb);
                    fma_step(acc, fa, fb);
                }
            }
            if (more) {
                store_tile(As[cur ^ 1], a_kc, tid, ra);
                store_tile(Bs[cur ^ 1], b_kc, tid, rb);
            }
            __syncthreads();
        }

#pragma unroll
        for (int i = 0; i < 16; i++) {
            const uint32_t m = m0 + ty * 4 + (i & 3) + 32 * (i >> 2);
            if (m >= a.M) continue;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t n = n0 + tx * 4 + (j & 3) + 64 * (j >> 2);
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
    // Groups of 4 start at multiples of 4 elements from the base (tile
    // origins, k0 and the thread offsets are all multiples of 4).
    const size_t esz = p.dtype == DT_F32 ? 4 : 2;
    auto vec_ok = [&](const void* base, uint32_t ld, int64_t stride) {
        return (reinterpret_cast<uintptr_t>(base) % (4 * esz)) == 0 && ld % 4 == 0 &&
               (p.batch == 1 || stride % 4 == 0);
    };
    a.vec_a = vec_ok(p.A, p.lda, p.sa) ? 1u : 0u;
    a.vec_b = vec_ok(p.B, p.ldb, p.sb) ? 1u : 0u;
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
