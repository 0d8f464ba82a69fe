// gemv.cu -- split-K decode GEMV for 2-byte types (M <= 16 rows of activations).
//
// Replaces the reference's decode family (lakitu12/vkblas src/vkblas.c:2501-2808,
// shaders matvec_splitk_tmpl.comp, matvec_splitk_m_tmpl.comp,
// splitk_reduce_half.comp, splitk_reduce_m_half.comp): C[m, n] = alpha *
// sum_k X[m, k] * W[n, k] + beta * C[m, n] for M <= 16, with W stored as
// N rows of K contiguous elements (the engine's op_b == T, i.e. hipBLAS
// transA == T on the weights -- test/bench_decode.c:52-64).  fp32 accumulate,
// fp32 epilogue, RNE store; split-K partial sums are added in segment order
// before the epilogue (splitk_reduce_half.comp:16-35).
//
// The kernel is HBM-bound on the weight stream (2*N*K bytes), so its design
// is about bytes in flight and resident warps:
//   - a CTA owns 16 weight rows; its 8 warps (4 when M > 8) split the K range
//     (intra-CTA split-K) and add their partial sums through shared memory
//     in warp order, so parallelism comes without global partials;
//   - every lane issues 128-bit loads of its rows straight into registers
//     (8 per 128-wide K step).  Shared-memory rings (cp.async, bulk copies,
//     2-D TMA) were measured slower here: the ring's footprint cut residency
//     to 8 warps per SM, too few to hide the per-warp load and MMA latency;
//   - the multiply runs on the tensor cores through mma.sync m16n8k16 (W rows
//     are the MMA's M, tokens its N) so that M = 16 is not FP32-bound; since
//     only the sum over k matters, each lane feeds the MMA the 8 consecutive k
//     it loaded (A and B see the same k permutation);
//   - optional inter-CTA split-K (gridDim.y segments) for short N: segment
//     partials go to a workspace and the last CTA of each row block (atomic
//     ticket, no waiting) reduces them in segment order, applies alpha/beta
//     and resets its ticket for the next launch.
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "vkblas_b200.h"

namespace vkb {
namespace {

// Warps per CTA (they split the CTA's K range).  A thread needs 61-64
// registers, so an SM holds 4 CTAs of 8 warps or 8 CTAs of 4 warps.  4-warp
// CTAs keep all 896 CTAs of a 14336-row layer resident in one wave (measured at
// M = 16: 27.0 us against 29.0 us with 8 warps); 8-warp CTAs give a short
// layer (few row blocks) more warps per row block.  See gemv_warps().
constexpr int ROWS_PER_CTA = 16;         // weight rows per CTA (one m16 MMA tile)
constexpr int KCHUNK = 64;

struct GemvArgs {
    const void* X; uint32_t ldx;          // M x K activations, k contiguous
    const void* W; uint32_t ldw;          // N x K weights, k contiguous
    void* C; uint32_t ldc;                // M x N output
    uint32_t M, N, K;
    uint32_t kspan;                       // K elements per segment (multiple of KCHUNK)
    uint32_t splitk;                      // segments (gridDim.y)
    float alpha, beta;
    const float* d_alpha;
    const float* d_beta;
    float* partial;                       // [splitk][M][N] fp32 (split-K only)
    unsigned* tickets;                    // [gridDim.x]   (split-K only)
    uint32_t k_rot;                       // k-step rotation multiplier (0 = plain order)
};

template <typename T> struct Mma;
template <> struct Mma<__half> {
    static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct Mma<__nv_bfloat16> {
    static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// Weights: read once -> bypass L1, 256-byte L2 fetches (a step reads 256
// contiguous bytes of each row).  Measured on B200 (4096 -> 14336, graph
// replay): with a 128-byte or no fetch hint M = 1 took 23.2 us instead of 20.7.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
// Activations: tiny and reused by every warp -> through L1.
__device__ __forceinline__ uint4 ldg_cached(const void* p) {
    uint4 v;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Two m16n8k16 steps covering 32 consecutive k (this lane's 8 of them are in
// w_lo (row g), w_hi (row g+8), x (token)): see the file comment.
template <typename T>
__device__ __forceinline__ void mma_32k(float (&d)[4], const uint4& w_lo, const uint4& w_hi,
                                        const uint4& x) {
    uint32_t a0[4] = {w_lo.x, w_hi.x, w_lo.y, w_hi.y};
    Mma<T>::run(d, a0, x.x, x.y);
    uint32_t a1[4] = {w_lo.z, w_hi.z, w_lo.w, w_hi.w};
    Mma<T>::run(d, a1, x.z, x.w);
}

template <typename T, bool TWO_NTILES, int KW>
__global__ void __launch_bounds__(KW * 32) gemv_kernel(GemvArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t nbase = blockIdx.x * ROWS_PER_CTA;
    const uint32_t seg = blockIdx.y;
    const uint32_t kbeg = seg * a.kspan;
    const uint32_t kend = min(a.K, kbeg + a.kspan);
    // This warp's slice of the segment (multiples of KCHUNK).
    const uint32_t per = ((kend - kbeg + KW - 1) / KW + KCHUNK - 1) / KCHUNK * KCHUNK;
    const uint32_t kw0 = min(kend, kbeg + (uint32_t)warp * per);
    const uint32_t kw1 = min(kend, kw0 + per);

    const T* W = reinterpret_cast<const T*>(a.W);
    const T* X = reinterpret_cast<const T*>(a.X);
    const uint32_t r0 = nbase + g, r1 = nbase + g + 8;
    const bool r0ok = r0 < a.N, r1ok = r1 < a.N;
    const uint32_t x0 = g, x1 = g + 8;                // tokens of n-tile 0 and 1
    const bool x0ok = x0 < a.M, x1ok = TWO_NTILES && x1 < a.M;
    const T* w0p = W + (size_t)(r0ok ? r0 : 0) * a.ldw;
    const T* w1p = W + (size_t)(r1ok ? r1 : 0) * a.ldw;
    const T* x0p = X + (size_t)(x0ok ? x0 : 0) * a.ldx;
    const T* x1p = X + (size_t)(x1ok ? x1 : 0) * a.ldx;

    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);

    // Two 64-wide chunks per step: 8 x 128-bit weight loads in flight per lane.
    // With k_rot != 0 the steps of CTA b start at step (b * k_rot) mod nstep and
    // wrap around, so that the CTAs do not all read the same k offset of their
    // rows at the same time.
    const uint32_t nstep = kw1 > kw0 ? (kw1 - kw0) / (2 * KCHUNK) : 0u;
    const uint32_t rot = (nstep && a.k_rot) ? (blockIdx.x * a.k_rot) % nstep : 0u;
    for (uint32_t i = 0; i < nstep; i++) {
        const uint32_t ii = i + rot < nstep ? i + rot : i + rot - nstep;
        const uint32_t kb = kw0 + ii * 2 * KCHUNK;
        uint4 w[2][2][2];                   // [chunk][half][row]
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t k = kb + c * KCHUNK + h * 32 + 8 * t;
                w[c][h][0] = r0ok ? ldg_stream(w0p + k) : z;
                w[c][h][1] = r1ok ? ldg_stream(w1p + k) : z;
            }
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t k = kb + c * KCHUNK + h * 32 + 8 * t;
                uint4 xa = x0ok ? ldg_cached(x0p + k) : z;
                mma_32k<T>(d0, w[c][h][0], w[c][h][1], xa);
                if (TWO_NTILES) {
                    uint4 xb = x1ok ? ldg_cached(x1p + k) : z;
                    mma_32k<T>(d1, w[c][h][0], w[c][h][1], xb);
                }
            }
    }
    // Tail: 32-wide halves; K is a multiple of 8, so each lane's 8-wide block
    // is entirely inside or entirely outside [kb, kw1).
    for (uint32_t kb = kw0 + nstep * 2 * KCHUNK; kb < kw1; kb += 32) {
        const uint32_t k = kb + 8 * t;
        const bool in = k < kw1;
        uint4 wl = (in && r0ok) ? ldg_stream(w0p + k) : z;
        uint4 wh = (in && r1ok) ? ldg_stream(w1p + k) : z;
        uint4 xa = (in && x0ok) ? ldg_cached(x0p + k) : z;
        mma_32k<T>(d0, wl, wh, xa);
        if (TWO_NTILES) {
            uint4 xb = (in && x1ok) ? ldg_cached(x1p + k) : z;
            mma_32k<T>(d1, wl, wh, xb);
        }
    }

    // Warp partials -> shared memory; warp 0 adds them in warp (= k) order.
    __shared__ float red[KW][TWO_NTILES ? 8 : 4][32];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        red[warp][i][lane] = d0[i];
        if (TWO_NTILES) red[warp][4 + i][lane] = d1[i];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float s0 = red[0][i][lane], s1 = TWO_NTILES ? red[0][4 + i][lane] : 0.f;
#pragma unroll
            for (int w = 1; w < KW; w++) {
                s0 = __fadd_rn(s0, red[w][i][lane]);
                if (TWO_NTILES) s1 = __fadd_rn(s1, red[w][4 + i][lane]);
            }
            d0[i] = s0;
            d1[i] = s1;
        }
    }

    float alpha = a.alpha, beta = a.beta;
    load_scalars(a.d_alpha, a.d_beta, alpha, beta);
    T* C = reinterpret_cast<T*>(a.C);

    // Fragment ownership: d[0]=(n=r0, m=2t) d[1]=(r0, 2t+1) d[2]=(r1, 2t) d[3]=(r1, 2t+1);
    // n-tile 1 adds 8 to m.
    if (a.splitk == 1) {
        if (warp != 0) return;
#pragma unroll
        for (int nt = 0; nt < (TWO_NTILES ? 2 : 1); nt++) {
            const float* d = nt ? d1 : d0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t n = (i < 2) ? r0 : r1;
                const uint32_t m = nt * 8 + 2 * t + (i & 1);
                if (n < a.N && m < a.M) {
                    T* cp = C + (size_t)m * a.ldc + n;
                    const float c = (beta != 0.f) ? Elem<T>::to_f(*cp) : 0.f;
                    *cp = Elem<T>::from_f(epilogue(alpha, d[i], beta, c));
                }
            }
        }
        return;
    }

    // Inter-CTA split-K: publish this segment's partials, then take a ticket.
    if (warp == 0) {
        float* P = a.partial + (size_t)seg * a.M * a.N;
#pragma unroll
        for (int nt = 0; nt < (TWO_NTILES ? 2 : 1); nt++) {
            const float* d = nt ? d1 : d0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t n = (i < 2) ? r0 : r1;
                const uint32_t m = nt * 8 + 2 * t + (i & 1);
                if (n < a.N && m < a.M) __stcg(P + (size_t)m * a.N + n, d[i]);
            }
        }
        __threadfence();
    }
    __syncthreads();
    __shared__ unsigned s_last;
    if (threadIdx.x == 0) {
        unsigned prev = atomicAdd(&a.tickets[blockIdx.x], 1u);
        s_last = (prev == a.splitk - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Last CTA of this row block: sum the partials in segment order.
    const uint32_t cells = (uint32_t)ROWS_PER_CTA * a.M;
    for (uint32_t e = threadIdx.x; e < cells; e += KW * 32) {
        const uint32_t m = e / ROWS_PER_CTA, n = nbase + e % ROWS_PER_CTA;
        if (n >= a.N) continue;
        float s = 0.f;
        for (uint32_t q = 0; q < a.splitk; q++)
            s = __fadd_rn(s, __ldcg(a.partial + ((size_t)q * a.M + m) * a.N + n));
        T* cp = C + (size_t)m * a.ldc + n;
        const float c = (beta != 0.f) ? Elem<T>::to_f(*cp) : 0.f;
        *cp = Elem<T>::from_f(epilogue(alpha, s, beta, c));
    }
    if (threadIdx.x == 0) a.tickets[blockIdx.x] = 0u;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint32_t gemv_kspan(uint32_t K, int splitk) {
    uint32_t span = (K + splitk - 1) / splitk;
    return (span + KCHUNK - 1) / KCHUNK * KCHUNK;
}

// Warps per CTA: 4 when M > 8 (two token tiles); for M <= 8, 8 unless the
// row-block CTAs of all segments would not fit in one wave of 4 such CTAs per
// SM, and then 4 (8 CTAs per SM).  VKBLAS_GEMV_WARPS=4|8 fixes it for M <= 8.
int gemv_warps(const GemmProblem& p, int splitk, int num_sms) {
    if (p.M > 8) return 4;
    static const int forced = [] {
        const char* e = getenv("VKBLAS_GEMV_WARPS");
        const int v = e ? atoi(e) : 0;
        return (v == 4 || v == 8) ? v : 0;
    }();
    if (forced) return forced;
    const uint64_t ctas = (uint64_t)((p.N + ROWS_PER_CTA - 1) / ROWS_PER_CTA) * (uint64_t)splitk;
    return ctas > 4ull * (uint64_t)num_sms ? 4 : 8;
}

// k-step rotation multiplier of the GEMV (VKBLAS_GEMV_KROT=n; 0 = plain order).
// In plain order all CTAs read the same k offset of their rows at the same
// time, and the HBM channels are unevenly loaded (ncu at M = 16: idlest
// channel 26.9% active, average 51.0%).  Measured on B200 at 4096 -> 14336
// (graph replay, one box): M = 1 22.3 -> 20.8 us, M = 8 22.65 -> 21.2 us,
// M = 16 23.8 -> 23.35 us with multiplier 3; multipliers 1, 5 and 7 gave the
// same within 0.1 us.
uint32_t gemv_k_rot() {
    static const uint32_t r = [] {
        const char* e = getenv("VKBLAS_GEMV_KROT");
        const int v = e ? atoi(e) : 3;
        return (uint32_t)(v < 0 ? 0 : v);
    }();
    return r;
}

int device_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return sms;
}

template <typename T>
void launch_typed(dim3 grid, bool two, int kw, const GemvArgs& a, cudaStream_t s) {
    if (two) gemv_kernel<T, true, 4><<<grid, 4 * 32, 0, s>>>(a);
    else if (kw == 4) gemv_kernel<T, false, 4><<<grid, 4 * 32, 0, s>>>(a);
    else gemv_kernel<T, false, 8><<<grid, 8 * 32, 0, s>>>(a);
}

// One launch over segments [0, segs) with the given partial/ticket areas
// (both unused when a single segment results).
cudaError_t launch_segments(const GemmProblem& p, int splitk, float* partial, unsigned* tickets,
                            cudaStream_t s) {
    if (splitk < 1) splitk = 1;
    uint32_t kspan = gemv_kspan(p.K, splitk);
    uint32_t segs = (p.K + kspan - 1) / kspan;        // may be < splitk after rounding
    if (segs < 1) segs = 1;
    if (segs > 1 && (!partial || !tickets)) return cudaErrorInvalidValue;
    GemvArgs a;
    a.X = p.A; a.ldx = p.lda; a.W = p.B; a.ldw = p.ldb; a.C = p.C; a.ldc = p.ldc;
    a.M = p.M; a.N = p.N; a.K = p.K; a.kspan = kspan; a.splitk = segs;
    a.alpha = p.alpha; a.beta = p.beta; a.d_alpha = p.d_alpha; a.d_beta = p.d_beta;
    a.partial = segs > 1 ? partial : nullptr;
    a.tickets = segs > 1 ? tickets : nullptr;
    a.k_rot = gemv_k_rot();
    dim3 grid((p.N + ROWS_PER_CTA - 1) / ROWS_PER_CTA, segs);
    const bool two = p.M > 8;
    const int kw = gemv_warps(p, (int)segs, device_sms());
    if (p.dtype == DT_F16) launch_typed<__half>(grid, two, kw, a, s);
    else if (p.dtype == DT_BF16) launch_typed<__nv_bfloat16>(grid, two, kw, a, s);
    else return cudaErrorInvalidValue;
    count_launch();
    return cudaGetLastError();
}

}  // namespace

bool gemv_supported(const GemmProblem& p) {
    return (p.dtype == DT_F16 || p.dtype == DT_BF16) && p.M >= 1 && p.M <= 16 && p.op_a == 0 &&
           p.op_b == 1 && p.batch == 1 && p.K % 8 == 0 && p.lda % 8 == 0 && p.ldb % 8 == 0 &&
           aligned16(p.A) && aligned16(p.B);
}

int gemv_auto_splitk(const GemmProblem& p, int num_sms) {
    // The warps of a CTA already split K; cut K across CTAs too only when
    // there are too few row blocks to keep every SM busy: aim at 24 resident
    // warps per SM (3 CTAs of 8 warps, or 6 of 4).  4-warp CTAs (8 per SM)
    // also keep the grid within one wave.  Measured at M = 16 against the 8-warp target alone:
    // 4096 rows x K = 14336 32.6 -> 24.3 us, 4096 x 4096 13.4 -> 12.1 us;
    // without the wave cap 11008 x 4096 went from 20.5 to 26.4 us.
    const uint32_t kw = (uint32_t)gemv_warps(p, 1, num_sms);
    const uint32_t target = (24u / kw) * (uint32_t)num_sms;
    const uint32_t wave = (32u / kw) * (uint32_t)num_sms;     // resident CTAs, all SMs
    const uint32_t ctas = (p.N + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
    int s = 1;
    while (s < 16 && ctas * s < target && p.K / (2u * s) >= kw * 128u &&
           (kw == 8 || ctas * 2u * s <= wave))
        s *= 2;
    return s;
}

// Workspace layout: [tickets: MAX_TICKETS x u32, zero on entry and left zero
// by the kernel][partials: splitk x M x N fp32].  The ticket area has a fixed
// size so that calls with different shapes never see each other's partials
// where they expect a zero ticket.
constexpr size_t MAX_TICKETS = 65536;
constexpr size_t TICKET_BYTES = MAX_TICKETS * sizeof(unsigned);

size_t gemv_workspace_bytes(const GemmProblem& p, int splitk) {
    if (splitk <= 1) return 0;
    return TICKET_BYTES + (size_t)splitk * p.M * p.N * sizeof(float);
}

cudaError_t launch_gemv(const GemmProblem& p, int splitk, void* workspace, int* d_status,
                        cudaStream_t s) {
    (void)d_status;     // this kernel never waits on another CTA
    const uint32_t ctas = (p.N + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
    if (splitk > 1 && (ctas > MAX_TICKETS || !workspace)) splitk = 1;
    unsigned* tickets = reinterpret_cast<unsigned*>(workspace);
    float* partial = workspace ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                                          TICKET_BYTES)
                               : nullptr;
    return launch_segments(p, splitk, partial, tickets, s);
}

}  // namespace vkb

// ---------------------------------------------------------------------------
// Split-K GEMV with library-owned scratch: vkblas_gemv_splitk_noalloc.
//
// Some callers cannot let a library call cudaMalloc: code that runs inside a
// framework's own memory pool or allocator hook (a nested cudaMalloc there can
// re-enter the allocator or bypass its accounting), and latency-critical
// decode loops, where the grow-only workspace behind vkblas_gemm_f16 may free
// and reallocate when a larger shape appears -- and cudaFree / cudaMalloc
// synchronise the whole device.  This entry point runs the same split-K GEMV
// kernel, but its scratch (split-K partial sums and per-row-block tickets)
// is the fixed array below, compiled into the library: it allocates nothing.
//
// Limits and sharing rules:
//   - the array holds kNoAllocScratchBytes = 4 MiB on every GPU that loads the
//     library, until the process exits;
//   - split-K partials need splitk * M * N * 4 bytes of the
//     kNoAllocPartialBytes part, and the kernel needs one ticket per 16 weight
//     rows of the kNoAllocTickets available; larger calls are rejected with
//     VKBLAS_ERR_PARAM before anything is enqueued;
//   - every call on a device shares the one array and it keeps the last
//     call's contents, so each call first clears the tickets it will use on
//     its stream; two calls whose kernels overlap on the GPU (different
//     streams, no ordering between them) race on the array and give wrong
//     results -- order such calls on one stream or with events;
//   - the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call
//     before any stream capture.
constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocTickets = 16384;
constexpr size_t kNoAllocTicketBytes = kNoAllocTickets * sizeof(unsigned);
constexpr size_t kNoAllocPartialBytes = kNoAllocScratchBytes - kNoAllocTicketBytes;

static __device__ __align__(256) unsigned char g_gemv_noalloc_scratch[kNoAllocScratchBytes];

namespace vkb {
namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on `dev` (the current device), looked up
// once per device.  The host-side symbol itself is only a stand-in: passing it
// to a kernel would fault or silently address host memory.
void* noalloc_scratch(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_gemv_noalloc_scratch) != cudaSuccess || !ptr) {
            cudaGetLastError();
            return nullptr;
        }
        g_noalloc_ptr[dev] = ptr;
    }
    return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace vkb

extern "C" __attribute__((visibility("default"))) vkblas_status_t vkblas_gemv_splitk_noalloc(
    vkblas_dtype_t dtype, uint32_t M, uint32_t N, uint32_t K, float alpha, const void* X,
    uint32_t ldx, const void* W, uint32_t ldw, float beta, void* C, uint32_t ldc,
    uint32_t splitk, void* stream) {
    using namespace vkb;
    if (dtype != VKBLAS_DT_F16 && dtype != VKBLAS_DT_BF16) return VKBLAS_ERR_PARAM;
    if (M == 0 || N == 0 || K == 0 || !X || !W || !C || splitk < 1 || splitk > 16)
        return VKBLAS_ERR_PARAM;
    GemmProblem p;
    p.dtype = dtype == VKBLAS_DT_F16 ? DT_F16 : DT_BF16;
    p.op_a = 0;
    p.op_b = 1;
    p.M = M; p.N = N; p.K = K;
    p.alpha = alpha; p.beta = beta;
    p.d_alpha = nullptr; p.d_beta = nullptr;
    p.A = X; p.lda = ldx; p.B = W; p.ldb = ldw; p.C = C; p.ldc = ldc;
    p.batch = 1; p.sa = 0; p.sb = 0; p.sc = 0;
    if (!gemv_supported(p)) return VKBLAS_ERR_PARAM;            // M <= 16, 16-byte alignment
    const size_t ctas = (N + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
    if ((size_t)splitk * M * N * sizeof(float) > kNoAllocPartialBytes || ctas > kNoAllocTickets)
        return VKBLAS_ERR_PARAM;                                 // beyond the fixed scratch
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    unsigned char* scratch = static_cast<unsigned char*>(noalloc_scratch(dev));
    if (!scratch) return VKBLAS_ERR_INIT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The kernel expects zero tickets (it leaves them zero), and the array keeps
    // whatever the last call left: clear the ones this call uses.
    if (splitk > 1 && cudaMemsetAsync(scratch, 0, ctas * sizeof(unsigned), s) != cudaSuccess) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    // Array layout: [tickets: kNoAllocTicketBytes][partials: kNoAllocPartialBytes].
    cudaError_t e = launch_segments(p, (int)splitk,
                                    reinterpret_cast<float*>(scratch + kNoAllocTicketBytes),
                                    reinterpret_cast<unsigned*>(scratch), s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e == cudaErrorInvalidValue ? VKBLAS_ERR_PARAM : VKBLAS_ERR_INIT;
    }
    return VKBLAS_OK;
}
