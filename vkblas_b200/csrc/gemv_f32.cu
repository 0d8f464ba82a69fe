// gemv_f32.cu -- fp32 decode GEMV (M <= 8 rows of activations).
//
// Replaces the reference's fp32 matvec (lakitu12/vkblas src/vkblas.c:3120-3161,
// shader matvec_f32_tmpl.comp, split-K reduce splitk_reduce_f32.comp):
// C[m, n] = alpha * sum_k X[m, k] * W(k, n) + beta * C[m, n] for the engine's
// op_a == N (X rows are K contiguous), batch 1, in two weight layouts:
//
//   - K x N weights (engine op_b == N; matvec_f32_tmpl.comp TB=0): a thread
//     owns 4 consecutive outputs and walks its K segment in order with fmaf,
//     reading 128-bit rows of W that the warp's lanes cover contiguously.
//     K is cut into S segments of ceil(K / S) across gridDim.y; the last CTA
//     of each column block (atomic ticket, no waiting) adds the segment sums
//     in segment order from +0 and applies alpha/beta.  That is exactly the
//     fp32 split-K model, so results are bit-identical to it for every S.
//   - N x K weights (engine op_b == T, i.e. hipBLAS transA == T weights;
//     TB=1): a warp owns 4 weight rows; its lanes read 128-bit chunks that
//     interleave along K (each warp load is 512 contiguous bytes of a row),
//     keep per-lane fp32 sums and add them with a fixed butterfly.  The
//     reference's own TB=1 grouping (4 products per step, contraction left
//     to the driver) is not reproducible bit for bit either; this one is
//     deterministic and checked against double.
//
// Both are HBM-bound on the 4*N*K weight bytes.  The exact sequential SIMT
// kernel stays available (VKBLAS_SGEMM=ffma, HIPBLAS_COMPUTE_32F_PEDANTIC).
#include "common.cuh"

namespace vkb {
namespace {

constexpr int MT_MAX = 8;                  // tokens
constexpr int KN_THREADS = 128;            // K x N kernel: 4 outputs per thread
constexpr uint32_t KN_COLS = KN_THREADS * 4;
constexpr int NK_WARPS = 8;                // N x K kernel: 4 rows per warp
constexpr uint32_t NK_ROWS = NK_WARPS * 4;
constexpr size_t MAX_TICKETS = 65536;      // shared GEMV workspace layout
constexpr size_t TICKET_BYTES = MAX_TICKETS * sizeof(unsigned);

struct F32Args {
    const float* X; uint32_t ldx;
    const float* W; uint32_t ldw;
    float* C; uint32_t ldc;
    uint32_t M, N, K;
    uint32_t kspan, splitk;
    float alpha, beta;
    const float* d_alpha;
    const float* d_beta;
    float* partial;                        // [splitk][M][N] (split only)
    unsigned* tickets;                     // [gridDim.x] (split only)
};

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float4 ld_stream4(const float* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

// After this CTA published its segment sums: take the block's ticket.  True
// in the CTA that arrived last, which then adds every segment in order (all
// partials of the block are in the workspace by then).
__device__ __forceinline__ bool split_arrive(const F32Args& a, unsigned* s_last) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&a.tickets[blockIdx.x], 1u);
        *s_last = (prev == a.splitk - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!*s_last) return false;
    __threadfence();
    return true;
}

__device__ __forceinline__ void store_out(const F32Args& a, uint32_t m, uint32_t n, float s,
                                          float alpha, float beta) {
    float* c = a.C + (size_t)m * a.ldc + n;
    const float old = (beta != 0.f) ? *c : 0.f;
    *c = epilogue(alpha, s, beta, old);
}

// Segment sums of column n (all tokens) in order from +0, then the epilogue.
__device__ __forceinline__ void finish_col(const F32Args& a, uint32_t m, uint32_t n, float alpha,
                                           float beta) {
    float s = 0.f;
    for (uint32_t q = 0; q < a.splitk; q++)
        s = __fadd_rn(s, __ldcg(a.partial + ((size_t)q * a.M + m) * a.N + n));
    store_out(a, m, n, s, alpha, beta);
}

// ------------------------------------------------------------- K x N weights
template <int MT>
__global__ void __launch_bounds__(KN_THREADS) gemv_f32_kn_kernel(F32Args a) {
    const uint32_t n0 = blockIdx.x * KN_COLS + threadIdx.x * 4;
    const uint32_t kb = blockIdx.y * a.kspan;
    const uint32_t ke = min(a.K, kb + a.kspan);
    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[m][i] = 0.f;
    const uint32_t M = min(a.M, (uint32_t)MT);
    if (n0 + 3 < a.N) {
        const float* w = a.W + n0;
#pragma unroll 8
        for (uint32_t k = kb; k < ke; k++) {
            const float4 v = ld_stream4(w + (size_t)k * a.ldw);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if ((uint32_t)m < M) {
                    const float x = __ldg(a.X + (size_t)m * a.ldx + k);
                    acc[m][0] = __fmaf_rn(x, v.x, acc[m][0]);
                    acc[m][1] = __fmaf_rn(x, v.y, acc[m][1]);
                    acc[m][2] = __fmaf_rn(x, v.z, acc[m][2]);
                    acc[m][3] = __fmaf_rn(x, v.w, acc[m][3]);
                }
            }
        }
    } else if (n0 < a.N) {                  // ragged last columns: scalar loads
        for (uint32_t k = kb; k < ke; k++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (n0 + i < a.N) {
                    const float wv = __ldg(a.W + (size_t)k * a.ldw + n0 + i);
#pragma unroll
                    for (int m = 0; m < MT; m++)
                        if ((uint32_t)m < M)
                            acc[m][i] = __fmaf_rn(__ldg(a.X + (size_t)m * a.ldx + k), wv, acc[m][i]);
                }
            }
        }
    }
    float alpha = a.alpha, beta = a.beta;
    load_scalars(a.d_alpha, a.d_beta, alpha, beta);
    if (a.splitk == 1) {
#pragma unroll
        for (int m = 0; m < MT; m++)
#pragma unroll
            for (int i = 0; i < 4; i++)
                if ((uint32_t)m < M && n0 + i < a.N)
                    store_out(a, m, n0 + i, __fadd_rn(0.f, acc[m][i]), alpha, beta);
        return;
    }
    float* P = a.partial + (size_t)blockIdx.y * a.M * a.N;
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++)
            if ((uint32_t)m < M && n0 + i < a.N) __stcg(P + (size_t)m * a.N + n0 + i, acc[m][i]);
    __shared__ unsigned s_last;
    if (!split_arrive(a, &s_last)) return;
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int i = 0; i < 4; i++)
            if ((uint32_t)m < M && n0 + i < a.N) finish_col(a, m, n0 + i, alpha, beta);
    if (threadIdx.x == 0) a.tickets[blockIdx.x] = 0u;
}

// ------------------------------------------------------------- N x K weights
template <int MT>
__global__ void __launch_bounds__(NK_WARPS * 32) gemv_f32_nk_kernel(F32Args a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t r0 = blockIdx.x * NK_ROWS + warp * 4;
    const uint32_t kb = blockIdx.y * a.kspan;
    const uint32_t ke = min(a.K, kb + a.kspan);
    const uint32_t M = min(a.M, (uint32_t)MT);
    float acc[4][MT];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[r][m] = 0.f;
    const float* wr[4];
#pragma unroll
    for (int r = 0; r < 4; r++) wr[r] = a.W + (size_t)min(r0 + r, a.N - 1) * a.ldw;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    // K is a multiple of 4 and kspan a multiple of 128: each lane's float4 is
    // wholly inside or outside [kb, ke).
    for (uint32_t k = kb + 4 * lane; k < ke; k += 256) {
        float4 w[2][4];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const uint32_t kk = k + 128 * h;
                w[h][r] = (kk < ke && r0 + r < a.N) ? ld_stream4(wr[r] + kk) : z;
            }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t kk = k + 128 * h;
            if (kk >= ke) break;
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if ((uint32_t)m < M) {
                    const float4 x = __ldg(reinterpret_cast<const float4*>(a.X + (size_t)m * a.ldx + kk));
#pragma unroll
                    for (int r = 0; r < 4; r++) {
                        float t = acc[r][m];
                        t = __fmaf_rn(x.x, w[h][r].x, t);
                        t = __fmaf_rn(x.y, w[h][r].y, t);
                        t = __fmaf_rn(x.z, w[h][r].z, t);
                        t = __fmaf_rn(x.w, w[h][r].w, t);
                        acc[r][m] = t;
                    }
                }
            }
        }
    }
    // Fixed butterfly over the 32 lanes (every lane ends with the same sum).
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int m = 0; m < MT; m++)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                acc[r][m] = __fadd_rn(acc[r][m], __shfl_xor_sync(0xffffffffu, acc[r][m], o));
    float alpha = a.alpha, beta = a.beta;
    load_scalars(a.d_alpha, a.d_beta, alpha, beta);
    // Lane r * MT + m owns output (m, r0 + r).
    float mine = 0.f;
    int rr = -1, mm = -1;
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int m = 0; m < MT; m++)
            if (lane == r * MT + m) { mine = acc[r][m]; rr = r; mm = m; }
    const bool owns = rr >= 0 && (uint32_t)mm < M && r0 + rr < a.N;
    if (a.splitk == 1) {
        if (owns) store_out(a, mm, r0 + rr, mine, alpha, beta);
        return;
    }
    if (owns) __stcg(a.partial + ((size_t)blockIdx.y * a.M + mm) * a.N + r0 + rr, mine);
    __shared__ unsigned s_last;
    if (!split_arrive(a, &s_last)) return;
    if (owns) finish_col(a, mm, r0 + rr, alpha, beta);
    if (threadIdx.x == 0) a.tickets[blockIdx.x] = 0u;
}

uint32_t blocks_x(const GemmProblem& p) {
    return p.op_b == 0 ? (p.N + KN_COLS - 1) / KN_COLS : (p.N + NK_ROWS - 1) / NK_ROWS;
}

uint32_t kspan_of(const GemmProblem& p, int splitk) {
    uint32_t span = (p.K + splitk - 1) / splitk;
    if (p.op_b == 1) span = (span + 127) / 128 * 128;     // whole 128-k lane steps
    return span;
}

template <int MT>
void launch_mt(const GemmProblem& p, const F32Args& a, dim3 grid, cudaStream_t s) {
    if (p.op_b == 0)
        gemv_f32_kn_kernel<MT><<<grid, KN_THREADS, 0, s>>>(a);
    else
        gemv_f32_nk_kernel<MT><<<grid, NK_WARPS * 32, 0, s>>>(a);
}

}  // namespace

bool gemv_f32_supported(const GemmProblem& p) {
    if (p.dtype != DT_F32 || p.M < 1 || p.M > (uint32_t)MT_MAX || p.op_a != 0 || p.batch != 1)
        return false;
    if (p.op_b == 0) return p.ldb % 4 == 0 && al16(p.B);
    return p.K % 4 == 0 && p.ldb % 4 == 0 && p.lda % 4 == 0 && al16(p.A) && al16(p.B);
}

int gemv_f32_auto_splitk(const GemmProblem& p, int num_sms) {
    const uint32_t bx = blocks_x(p);
    // CTAs to keep every SM streaming: a K x N thread has one 16-byte row load
    // per k in flight (unrolled 8), so that kernel wants three times as many
    // of its 4-warp CTAs as the 8-warp N x K kernel.
    const uint32_t want = (p.op_b == 0 ? 12u : 4u) * (uint32_t)num_sms;
    if (bx >= want) return 1;
    uint32_t s = (want + bx - 1) / bx;
    const uint32_t min_span = p.op_b == 0 ? 64u : 512u;
    if (s > p.K / min_span) s = p.K / min_span;
    if (s > 64) s = 64;
    return s < 1 ? 1 : (int)s;
}

size_t gemv_f32_workspace_bytes(const GemmProblem& p, int splitk) {
    if (splitk <= 1) return 0;
    return TICKET_BYTES + (size_t)splitk * p.M * p.N * sizeof(float);
}

cudaError_t launch_gemv_f32(const GemmProblem& p, int splitk, void* workspace, cudaStream_t s) {
    if (splitk < 1) splitk = 1;
    if (splitk > 1 && (!workspace || blocks_x(p) > MAX_TICKETS)) splitk = 1;
    const uint32_t span = kspan_of(p, splitk);
    const uint32_t segs = (p.K + span - 1) / span;
    F32Args a;
    a.X = reinterpret_cast<const float*>(p.A); a.ldx = p.lda;
    a.W = reinterpret_cast<const float*>(p.B); a.ldw = p.ldb;
    a.C = reinterpret_cast<float*>(p.C); a.ldc = p.ldc;
    a.M = p.M; a.N = p.N; a.K = p.K;
    a.kspan = span; a.splitk = segs;
    a.alpha = p.alpha; a.beta = p.beta; a.d_alpha = p.d_alpha; a.d_beta = p.d_beta;
    a.tickets = segs > 1 ? reinterpret_cast<unsigned*>(workspace) : nullptr;
    a.partial = segs > 1 ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + TICKET_BYTES)
                         : nullptr;
    const dim3 grid(blocks_x(p), segs);
    if (p.M <= 1) launch_mt<1>(p, a, grid, s);
    else if (p.M <= 2) launch_mt<2>(p, a, grid, s);
    else if (p.M <= 4) launch_mt<4>(p, a, grid, s);
    else launch_mt<8>(p, a, grid, s);
    count_launch();
    return cudaGetLastError();
}

}  // namespace vkb
