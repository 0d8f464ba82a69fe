// umma_gemm.cu -- tcgen05 (5th-gen tensor core) GEMM for sm_100a.
//
// Replaces the reference's tile shaders for the large-GEMM path (lakitu12/vkblas
// src/shaders/gemm_half_128x128_bankfree_tmpl.comp, gemm_f32_128x128_bankfree_tmpl.comp
// and their 64x64 / 128x256 / split-K variants, dispatched from
// src/vkblas.c:1550-1756 and 2810-2884).  Same contract: row-major
// C = alpha*op(A)*op(B) + beta*C per batch entry, fp32 accumulation, fp32
// epilogue with C unread when beta == 0, RNE store for 2-byte outputs.
//
// Structure (one CTA per SM, or one 2-CTA cluster per SM pair for 256-row
// tiles, persistent over output tiles):
//   warp 0      TMA producer: SWIZZLE_128B tiles of A and B into a STAGES-deep
//               shared-memory ring (full/empty mbarrier pairs); a stage holds
//               KBS consecutive k-blocks.  op(A)/op(B) are absorbed here: a
//               K-major operand is loaded as rows of 128 bytes of K, an
//               MN-major one as 128-byte slabs of M (or N) per k-row, and the
//               UMMA descriptors say which (no transpose pass, unlike the
//               reference's transpose shaders, src/vkblas.c:970-1188).
//   warp 1      allocates TMEM (two accumulators, double-buffered across
//               tiles) and issues tcgen05.mma from one thread; tcgen05.commit
//               releases smem stages and hands finished accumulators over.
//   warps 2-5   epilogue (2-9 for 3xTF32): tcgen05.ld (32 lanes x 32 columns
//               per step) -> alpha/beta -> convert -> global, overlapping the
//               next tile's main loop.  2-byte C goes through 32 x 64 boxes in
//               shared memory and TMA stores (to peer copies of C as well).
// 2-byte GEMMs are launched as programmatic dependents of the previous kernel
// on the stream; every global access waits in griddepcontrol.wait first.
// Long fp16/bf16 pair grids may run their last wave as 256 x 128 halves in a
// second, dependent grid (the narrow tail, unit_coords).
//
// fp32 (3xTF32, after Ootomo & Yokota 2022, "Recovering single precision
// accuracy from Tensor Cores while surpassing the FP32 theoretical peak
// performance"): a pre-pass splits each operand x into big = tf32(x) and
// small = tf32(x - big) (both round-to-nearest-even, low 13 bits zero, written
// as compact K-major planes in a workspace -- an MN-major operand is
// transposed on the way, the tf32 MMAs only ever read K-major tiles) and the
// main loop accumulates A_small*B_big + A_big*B_small + A_big*B_big into one
// fp32 TMEM accumulator.
//
// No TMA load uses cluster multicast: each CTA issues its own loads.  The only
// multicast is tcgen05.commit's, which signals both CTAs of a pair.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "umma.cuh"

namespace vkb {
namespace {

using namespace umma;

enum Kind : int { K_F16 = 0, K_BF16 = 1, K_TF32X3 = 2 };

constexpr int BM = 128;
constexpr uint32_t ROW_BYTES = 128;       // one SWIZZLE_128B atom row
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;       // 2 s
constexpr uint64_t TEST_WAIT_LIMIT_NS = 20000000ull;    // 20 ms when the test hook is on
constexpr uint64_t DRAIN_LIMIT_NS = 200000000ull;

struct __align__(64) UmmaParams {
    CUtensorMap tmA[2];          // [plane]; 2-byte kinds use plane 0, 3xTF32 big / small
    CUtensorMap tmB[2];
    // C as TMA store targets (c_tma): [0] this GPU's C, [1 + j] peer j's copy.
    // 32-row x 64-column boxes, SWIZZLE_128B, over [batch][M][N].
    CUtensorMap tmC[8];
    void* C;
    uint32_t ldc;
    int64_t sc;
    uint32_t M, N, K, batch;
    uint32_t tiles_m, tiles_n, num_kb, total_tiles;
    // Work units: tiles [0, full_tiles) whole; every later tile cut into
    // split_s K ranges of split_kb k-blocks (stream-K tail / split-K).
    uint32_t full_tiles, split_s, split_kb, total_units;
    float* partial;              // [(total_tiles - full_tiles) * split_s][BN][BM] fp32
    uint32_t a_batched, b_batched;
    float alpha, beta;
    const float* d_alpha;
    const float* d_beta;
    int* status;
    uint32_t c_vec_ok;
    // C transposed: the kernel computes C^T = op(B)^T op(A)^T (small-M decode
    // shapes, weight rows on the MMA's 128 lanes) and element (row, col) of
    // its tile goes to C + col * ldc + row.
    uint32_t c_trans;
    // k-block order rotation (small-M tiles only): a unit of tile t starts its
    // k range at (t * k_rot_mul) % len and wraps around (0 = plain order).
    uint32_t k_rot_mul;
    uint64_t wait_limit_ns;      // bound of every mbarrier wait
    uint32_t test_skip_first_load;   // test hook: the first stage is never filled
    uint32_t mma_group;          // stages the MMA issuer takes at a time; 0 = Cfg::MMA_GROUP
    // Replicated C: every value written to C is also written, at the same
    // element offset from C, to each of the npeers copies (other GPUs' C
    // buffers mapped into this process; the stores cross NVLink).
    void* peer[7];
    uint32_t npeers;
    // 1: the epilogue stages whole C boxes in shared memory and stores them
    // with TMA (2-byte kinds whose C TMA can describe; see Cfg::EPI_STAGE).
    uint32_t c_tma;
    // Narrow tail (half-width launch of a 256-wide grid's last tiles): unit u
    // is half (u & 1) of tile tail_first + (u >> 1) of the 256-wide tile grid
    // (tiles_m x tiles_n); NO_TAIL otherwise.
    uint32_t tail_first;
    uint32_t group_m;            // M-blocks that sweep the N-blocks together (tile order)
    // 1: this grid reads nothing the previous grid writes before it ends (the
    // narrow tail after its main launch), so it waits for that grid only at
    // its end, and so finishes after it.
    uint32_t dep_end;
};
constexpr uint32_t NO_TAIL = 0xFFFFFFFFu;

template <typename V, typename T>
__device__ __forceinline__ void put_c(const UmmaParams& p, T* c, size_t off, const V& val) {
    *reinterpret_cast<V*>(c) = val;
    for (uint32_t j = 0; j < p.npeers; j++)
        *reinterpret_cast<V*>(reinterpret_cast<T*>(p.peer[j]) + off) = val;
}

template <int KIND> struct OutT;
template <> struct OutT<K_F16> { using T = __half; };
template <> struct OutT<K_BF16> { using T = __nv_bfloat16; };
template <> struct OutT<K_TF32X3> { using T = float; };

__device__ __forceinline__ void tile_coords(const UmmaParams& p, uint32_t t, uint32_t& b,
                                            uint32_t& mb, uint32_t& nb) {
    const uint32_t per = p.tiles_m * p.tiles_n;
    b = t / per;
    const uint32_t r = t - b * per;
    // Groups of group_m M-blocks sweep the N-blocks together: consecutive tiles
    // (which run concurrently on neighbouring SMs) share A rows and B columns in L2.
    const uint32_t G = p.group_m;
    const uint32_t group = r / (G * p.tiles_n);
    const uint32_t first_m = group * G;
    const uint32_t gsize = min(p.tiles_m - first_m, G);
    const uint32_t in = r - group * G * p.tiles_n;
    mb = first_m + in % gsize;
    nb = in / gsize;
}

// Epilogue of 32 consecutive outputs of one row: C = alpha*v + beta*C (C not
// read when beta == 0), converted to T; 128-bit accesses when aligned.
constexpr uint32_t NO_SPLIT = 0xFFFFFFFFu;

// Work unit u -> (tile, split index or NO_SPLIT, k-block range).
__device__ __forceinline__ void unit_info(const UmmaParams& p, uint32_t u, uint32_t& tile,
                                          uint32_t& sp, uint32_t& kb0, uint32_t& kb1) {
    if (u < p.full_tiles) {
        tile = u;
        sp = NO_SPLIT;
        kb0 = 0;
        kb1 = p.num_kb;
    } else {
        const uint32_t v = u - p.full_tiles;
        tile = p.full_tiles + v / p.split_s;
        sp = v % p.split_s;
        kb0 = sp * p.split_kb;
        kb1 = min(p.num_kb, kb0 + p.split_kb);
    }
}

// `off`: element offset of crow from C (the same offset in every peer copy).
// Unit w -> its tile t (split bookkeeping), K range and C coordinates; in a
// narrow-tail grid the column block counts BN-wide blocks of the half tiles.
__device__ __forceinline__ void unit_coords(const UmmaParams& p, uint32_t w, uint32_t& t,
                                            uint32_t& sp, uint32_t& kb0, uint32_t& kb1,
                                            uint32_t& b, uint32_t& mb, uint32_t& nb) {
    unit_info(p, w, t, sp, kb0, kb1);
    if (p.tail_first != NO_TAIL) {
        tile_coords(p, p.tail_first + (w >> 1), b, mb, nb);
        nb = nb * 2u + (w & 1u);
    } else {
        tile_coords(p, t, b, mb, nb);
    }
}

template <typename T>
__device__ __forceinline__ void store_row32(const UmmaParams& p, T* crow, size_t off,
                                            const float (&v)[32], uint32_t ncols, bool vec,
                                            float alpha, float beta) {
    if (vec && ncols == 32) {
        if constexpr (sizeof(T) == 2) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                uint4 old = make_uint4(0, 0, 0, 0);
                if (beta != 0.f) old = *reinterpret_cast<const uint4*>(crow + q * 8);
                const T* o = reinterpret_cast<const T*>(&old);
                uint4 out;
                T* w = reinterpret_cast<T*>(&out);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float c = (beta != 0.f) ? Elem<T>::to_f(o[i]) : 0.f;
                    w[i] = Elem<T>::from_f(epilogue(alpha, v[q * 8 + i], beta, c));
                }
                put_c(p, crow + q * 8, off + q * 8, out);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 8; q++) {
                float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
                if (beta != 0.f) old = *reinterpret_cast<const float4*>(crow + q * 4);
                float4 out;
                out.x = epilogue(alpha, v[q * 4 + 0], beta, old.x);
                out.y = epilogue(alpha, v[q * 4 + 1], beta, old.y);
                out.z = epilogue(alpha, v[q * 4 + 2], beta, old.z);
                out.w = epilogue(alpha, v[q * 4 + 3], beta, old.w);
                put_c(p, crow + q * 4, off + q * 4, out);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) {
            if ((uint32_t)i < ncols) {
                const float c = (beta != 0.f) ? Elem<T>::to_f(crow[i]) : 0.f;
                put_c(p, crow + i, off + i, Elem<T>::from_f(epilogue(alpha, v[i], beta, c)));
            }
        }
    }
}

// Transposed epilogue: this thread's tile row `row` is a column of C, its 32
// values go down C's rows n0.. (lanes hold consecutive columns of C, so each
// store instruction of a warp is contiguous).
template <typename T>
__device__ __forceinline__ void store_col32(T* cb, uint32_t row, uint32_t n0, uint32_t ldc,
                                            const float (&v)[32], uint32_t ncols, float alpha,
                                            float beta) {
#pragma unroll
    for (int i = 0; i < 32; i++) {
        if ((uint32_t)i < ncols) {
            T* c = cb + (size_t)(n0 + i) * ldc + row;
            const float old = (beta != 0.f) ? Elem<T>::to_f(*c) : 0.f;
            *c = Elem<T>::from_f(epilogue(alpha, v[i], beta, old));
        }
    }
}

template <int KIND, bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR, int KBS = 1>
struct Cfg {
    static constexpr int E = (KIND == K_TF32X3) ? 4 : 2;
    static constexpr int PLANES = (KIND == K_TF32X3) ? 2 : 1;
    static constexpr int BK = ROW_BYTES / E;          // K elements per stage (64 or 32)
    static constexpr int UK = 32 / E;                 // K per UMMA instruction (16 or 8)
    static constexpr int KSTEPS = BK / UK;            // 4
    static constexpr int EPB = ROW_BYTES / E;         // elements per 128-byte MN slab
    // A CTA pair (PAIR) computes 256 x BN tiles: each CTA loads its 128 rows of
    // A and BN/2 columns of B.
    static constexpr int BM_TILE = PAIR ? 2 * BM : BM;
    static constexpr int BNC = PAIR ? BN / 2 : BN;             // B rows (N) per CTA
    static constexpr uint32_t A_PLANE = BM * ROW_BYTES;
    static constexpr uint32_t B_PLANE = BNC * ROW_BYTES;
    // A stage holds KBS consecutive k-blocks (each its A and B tiles, A
    // first), filled as one and released by one commit: the MMA issuer then
    // waits once and commits once per 4 * KBS MMAs.
    static constexpr uint32_t KB_BYTES = PLANES * (A_PLANE + B_PLANE);
    static constexpr uint32_t STAGE_BYTES = KBS * KB_BYTES;
    // The tensor core's fp32 accumulation truncates, so its error grows
    // linearly with the number of accumulating MMAs (measured on B200: relative
    // error ~7e-9 * K, biased toward zero).  3xTF32 therefore accumulates each
    // SEG_KB-block K segment in a fresh TMEM buffer and the epilogue adds the
    // segments in fp32 with round-to-nearest; 2-byte kinds keep one
    // accumulator per tile (their tolerance is far above that error).
    static constexpr uint32_t SEG_KB = (KIND == K_TF32X3) ? 8u : 0u;
    // TMEM accumulator buffers: 512 columns hold four 128-wide or two 256-wide.
    static constexpr uint32_t NBUF = (SEG_KB && BN <= 128) ? 4u : 2u;
    // Epilogue warps: 4 (one per TMEM lane quarter), or 8 for the segmented
    // epilogue, where two warps share a quarter and each keeps the fp32 sums of
    // half of the tile's columns in registers.
    static constexpr int EPI_WARPS = SEG_KB ? 8 : 4;
    static constexpr int EPI_COLS = BN * 4 / EPI_WARPS;          // columns per epilogue thread
    // A 256-wide segmented tile keeps 128 fp32 sums per epilogue thread, more
    // than an even share of the register file allows.  Its block has 12 warps:
    // warpgroup 0 (TMA producer, MMA issuer, two idle warps) drops to REGS_LOW
    // registers a thread and the two epilogue warpgroups rise to REGS_HIGH
    // (setmaxnreg).  The host launches it only when the split fits the
    // registers the block is launched with (launch_kind).
    static constexpr bool REG_SPLIT = SEG_KB != 0 && EPI_COLS > 64;
    static constexpr int EPI_WARP0 = REG_SPLIT ? 4 : 2;           // first epilogue warp
    static constexpr int THREADS = 32 * EPI_WARP0 + 32 * EPI_WARPS;
    static constexpr uint32_t REGS_LOW = 56, REGS_HIGH = 208;
    static constexpr uint32_t TMEM_COLS = NBUF * BN;                // 512
    // 2-byte tiles 128 or more wide can stage C in shared memory: each
    // epilogue warp fills 32-row x 64-column (128-byte rows, SWIZZLE_128B)
    // boxes, two in turn, and one lane stores each with TMA -- whole 128-byte
    // lines, also to peer copies over NVLink, instead of one 16-byte piece of
    // 32 different rows per store instruction.
    static constexpr bool EPI_STAGE = KIND != K_TF32X3 && BN >= 128;
    static constexpr uint32_t EPI_BOX = 32u * ROW_BYTES;
    static constexpr uint32_t EPI_BYTES = EPI_STAGE ? (uint32_t)EPI_WARPS * 2u * EPI_BOX : 0u;
    static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
    static constexpr uint32_t IDESC =
        instr_desc(KIND == K_F16 ? 0u : KIND == K_BF16 ? 1u : 2u, A_MN, B_MN, BM_TILE, BN);
    // Accumulator hand-back: every epilogue thread of the CTA (of both CTAs
    // for a pair, on the even CTA's barrier).
    static constexpr uint32_t TEMPTY_COUNT = (PAIR ? 2u : 1u) * 32u * EPI_WARPS;
    static constexpr uint32_t SLAB = BK * ROW_BYTES;  // MN-major: one 128-byte-wide slab
    // Stages the MMA issuer takes at a time (wait for all, one fence, all their
    // MMAs, one commit each).  Each stage costs a fixed 80-90 tensor cycles on
    // top of its MMAs, so rings deep enough to spare a stage of look-ahead take
    // two at a time.  Measured on B200 (one box, G = 1 -> 2): fp16 pair HGEMM
    // 4096^3 128.7 -> 117.8 us, 8192^3 915 -> 865 us, 256 x 2048^3 batched
    // 3928 -> 3715 us, small-M decode M = 16 33.5 -> 31.5 us; the 3-stage
    // 3xTF32 ring went 541 -> 703 us, so it keeps 1.
    static constexpr uint32_t MMA_GROUP = STAGES >= 6 ? 2u : 1u;
    static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
    static_assert(SEG_KB % KBS == 0, "a segment is whole stages");
    static_assert(MMA_GROUP >= 1, "the issuer takes at least one stage at a time");
    static_assert(KBS == 1 || (KIND != K_TF32X3 && SEG_KB == 0), "several k-blocks a stage: 2-byte kinds");
    static_assert(SEG_KB == 0 || EPI_COLS <= 128, "segmented epilogue keeps EPI_COLS fp32 sums per thread");
    static_assert(!REG_SPLIT || (REGS_LOW % 8 == 0 && REGS_HIGH % 8 == 0 && REGS_LOW >= 24 &&
                                 REGS_HIGH <= 256 && THREADS == 384),
                  "register split: one 128-thread warpgroup low, two high");
};

template <int KIND, bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR, int KBS = 1>
__global__ void __launch_bounds__(Cfg<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>::THREADS, 1)
    umma_gemm_kernel(const __grid_constant__ UmmaParams p) {
    using C_ = Cfg<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>;
    using TOut = typename OutT<KIND>::T;
    constexpr uint32_t NBUF = C_::NBUF;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (raw_base & 1023u)) & 1023u;
    uint8_t* smem = smem_raw + pad;
    const uint32_t sbase = raw_base + pad;
    const uint32_t epi_smem = sbase + STAGES * C_::STAGE_BYTES;     // 1024-aligned
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C_::STAGE_BYTES + C_::EPI_BYTES);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](uint32_t s) { return bar0 + 8u * s; };
    auto empty_bar = [&](uint32_t s) { return bar0 + 8u * (STAGES + s); };
    auto tfull_bar = [&](uint32_t a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](uint32_t a) { return bar0 + 8u * (2 * STAGES + NBUF + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 2 * NBUF);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NBUF + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pairs: rank 0 issues the MMAs; both CTAs' copies complete on its full
    // barriers and both CTAs' epilogues hand accumulators back on its tempty
    // barriers.  Work units are per pair.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool issuer = rank == 0;
    const uint32_t unit0 = PAIR ? blockIdx.x >> 1 : blockIdx.x;
    const uint32_t ustride = PAIR ? gridDim.x >> 1 : gridDim.x;
    auto to_issuer = [&](uint32_t bar) { return PAIR ? mapa_shared(bar, 0) : bar; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (uint32_t a = 0; a < NBUF; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), C_::TEMPTY_COUNT);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&p.tmA[0]);
        prefetch_tmap(&p.tmB[0]);
        if (C_::PLANES == 2) {
            prefetch_tmap(&p.tmA[1]);
            prefetch_tmap(&p.tmB[1]);
        }
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), C_::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C_::TMEM_COLS);
            tmem_relinquish();
        }
    }
    __syncthreads();
    if constexpr (PAIR) cluster_sync();      // the peer's barriers are initialised
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Warp roles.  With a register split, setmaxnreg opens each warpgroup's
    // branch, so that the compiler allocates each branch within its limit.
    if (warp < C_::EPI_WARP0) {
        if constexpr (C_::REG_SPLIT)
            asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C_::REGS_LOW));
        if (warp == 0) {
            // ------------------------------------------------------ TMA producer
            if (lane == 0) {
                // A 3xTF32 GEMM is the programmatic dependent of the split
                // pre-pass that writes its operand planes: wait for that grid
                // to finish and its writes to be visible before the first
                // load.  Nothing else of this kernel reads memory the pre-pass
                // writes.  Without a prerequisite grid this returns at once.
                if (!p.dep_end) asm volatile("griddepcontrol.wait;" ::: "memory");
                // Only now let a programmatic dependent (the next GEMM, a split
                // reduce, a narrow tail) launch: when it starts, every grid
                // before this one has finished, which a narrow tail relies on
                // to read A, B and C without waiting for this grid.
                asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
                uint32_t stage = 0, phase = 0;
                uint32_t issued_mask = 0, issued_parity = 0;   // per stage: issued ever / last parity
                bool ok = true;
                for (uint32_t u = unit0; ok && u < p.total_units; u += ustride) {
                    uint32_t t, sp, ukb0, ukb1, b, mb, nb;
                    unit_coords(p, u, t, sp, ukb0, ukb1, b, mb, nb);
                    const int32_t m0 = (int32_t)(mb * C_::BM_TILE + rank * BM);
                    const int32_t n0 = (int32_t)(nb * BN + rank * C_::BNC);
                    const int32_t ba = p.a_batched ? (int32_t)b : 0, bb = p.b_batched ? (int32_t)b : 0;
                    const uint32_t len = ukb1 - ukb0;
                    // Only the weight-streaming small-M tiles (BN = 64) rotate: all
                    // tiles start together, and in plain order every weight row
                    // would be read at the same k offset at the same time, which
                    // loads the HBM channels unevenly.
                    const uint32_t rot = (BN == 64 && p.k_rot_mul) ? (t * p.k_rot_mul) % len : 0u;
                    for (uint32_t i = 0; i < len; i += KBS) {
                        const uint32_t nk = min((uint32_t)KBS, len - i);   // k-blocks in this stage
                        if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag, p.status,
                                      DS_TIMEOUT_PRODUCER, p.wait_limit_ns)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = to_issuer(full_bar(stage));
                        if (p.test_skip_first_load && u == unit0 && i == 0) {
                            // Test hook: leave this stage empty so its consumer's
                            // bounded wait runs out (no copy is issued).
                            if (++stage == STAGES) {
                                stage = 0;
                                phase ^= 1u;
                            }
                            continue;
                        }
                        // The issuer expects both CTAs' bytes of a pair stage.
                        if (issuer)
                            mbar_arrive_expect_tx(full_bar(stage), (PAIR ? 2u : 1u) * nk * C_::KB_BYTES);
                        auto load = [&](uint32_t dst, const CUtensorMap* m, int32_t c0, int32_t c1,
                                        int32_t c2) {
                            if constexpr (PAIR) tma_load_3d_pair(dst, m, fb, c0, c1, c2);
                            else tma_load_3d(dst, m, fb, c0, c1, c2);
                        };
                        for (uint32_t sub = 0; sub < nk; sub++) {
                        const uint32_t ii = i + sub;
                        const uint32_t kb = ukb0 + (ii + rot < len ? ii + rot : ii + rot - len);
                        const uint32_t sA = sbase + stage * C_::STAGE_BYTES + sub * C_::KB_BYTES;
                        const uint32_t sB = sA + C_::PLANES * C_::A_PLANE;
                        const int32_t k0 = (int32_t)(kb * C_::BK);
#pragma unroll
                        for (int pl = 0; pl < C_::PLANES; pl++) {
                            if (!A_MN) {
                                load(sA + pl * C_::A_PLANE, &p.tmA[pl], k0, m0, ba);
                            } else {
#pragma unroll
                                for (int j = 0; j < BM / C_::EPB; j++)
                                    load(sA + pl * C_::A_PLANE + j * C_::SLAB, &p.tmA[pl],
                                         m0 + j * C_::EPB, k0, ba);
                            }
                            if (!B_MN) {
                                load(sB + pl * C_::B_PLANE, &p.tmB[pl], k0, n0, bb);
                            } else {
#pragma unroll
                                for (int j = 0; j < C_::BNC / C_::EPB; j++)
                                    load(sB + pl * C_::B_PLANE + j * C_::SLAB, &p.tmB[pl],
                                         n0 + j * C_::EPB, k0, bb);
                            }
                        }
                        }
                        issued_mask |= 1u << stage;
                        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
                // Never leave with copies in flight: wait for the last fill of every
                // stage (the issuer's full barrier; in the other CTA of a pair, the
                // stage's release by the issuer's MMAs, which follows its landing).
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        drain_bar_wait(issuer ? full_bar(s) : empty_bar(s), (issued_parity >> s) & 1u,
                                       p.status, DS_TIMEOUT_PRODUCER, DRAIN_LIMIT_NS);
            }
        } else if (warp == 1) {
            // ------------------------------------------------------- MMA issuer
            if (lane == 0 && issuer) {
                uint32_t stage = 0, phase = 0, u = 0;          // u: accumulator hand-overs so far
                bool ok = true;
                if constexpr (KBS > 1) {
                    // Whole units (2-byte kinds have no K segments), one stage of
                    // KBS k-blocks at a time: one wait, one fence, 4 * KBS MMAs,
                    // one commit.  Measured on B200: waiting for the next stage
                    // before the current stage's last k-block instead (so that
                    // queued MMAs cover the wait) was slower, 104.0 -> 111.2 us
                    // at 4096^3 and 755 -> 789 us at 8192^3, as the issuer then
                    // sometimes waits for data with MMAs still unissued.  So was
                    // waiting for the next stage between a stage's MMAs and its
                    // commit (100.4 -> 102.9 us and 744 -> 753 us).
                    for (uint32_t w = unit0; ok && w < p.total_units; w += ustride, u++) {
                        uint32_t t, sp, ukb0, ukb1;
                        unit_info(p, w, t, sp, ukb0, ukb1);
                        const uint32_t buf = u % NBUF, bph = (u / NBUF) & 1u;
                        if (!wait_bar(tempty_bar(buf), bph ^ 1u, abort_flag, p.status, DS_TIMEOUT_MMA,
                                      p.wait_limit_ns)) {
                            ok = false;
                            break;
                        }
                        const uint32_t d = tmem_base + buf * BN;
                        const uint32_t len = ukb1 - ukb0;
                        const uint32_t nst = (len + KBS - 1) / KBS;
                        tc_fence_after();
                        for (uint32_t si = 0; si < nst; si++) {
                            const uint32_t nk = min((uint32_t)KBS, len - si * KBS);
                            if (!wait_bar(full_bar(stage), phase, abort_flag, p.status, DS_TIMEOUT_MMA,
                                          p.wait_limit_ns)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            // Descriptors of this stage's first k-block; the others
                            // differ only in the start address field (bytes >> 4,
                            // which stays inside its 14 bits below 256 KB).
                            const uint32_t sA0 = sbase + stage * C_::STAGE_BYTES;
                            const uint64_t ad0 = A_MN ? smem_desc_sw128(sA0, C_::SLAB, 1024)
                                                      : smem_desc_sw128(sA0, 16, 1024);
                            const uint64_t bd0 = B_MN ? smem_desc_sw128(sA0 + C_::A_PLANE, C_::SLAB, 1024)
                                                      : smem_desc_sw128(sA0 + C_::A_PLANE, 16, 1024);
#pragma unroll
                            for (uint32_t sub = 0; sub < (uint32_t)KBS; sub++) {
                                if (sub >= nk) break;
#pragma unroll
                                for (int j = 0; j < C_::KSTEPS; j++) {
                                    constexpr uint32_t STEP = (A_MN ? C_::UK * ROW_BYTES : 32u) >> 4;
                                    constexpr uint32_t STEPB = (B_MN ? C_::UK * ROW_BYTES : 32u) >> 4;
                                    const uint64_t ad = ad0 + ((sub * C_::KB_BYTES) >> 4) + j * STEP;
                                    const uint64_t bd = bd0 + ((sub * C_::KB_BYTES) >> 4) + j * STEPB;
                                    const uint32_t first = (si == 0 && sub == 0 && j == 0) ? 0u : 1u;
                                    if constexpr (PAIR) mma_f16_pair(d, ad, bd, C_::IDESC, first);
                                    else mma_f16(d, ad, bd, C_::IDESC, first);
                                }
                            }
                            if constexpr (PAIR) tc_commit_pair_mc(empty_bar(stage), 0x3);
                            else tc_commit(empty_bar(stage));
                            if (++stage == STAGES) {
                                stage = 0;
                                phase ^= 1u;
                            }
                        }
                        if (!ok) break;
                        if constexpr (PAIR) tc_commit_pair_mc(tfull_bar(buf), 0x3);    // both epilogues
                        else tc_commit(tfull_bar(buf));
                    }
                } else {
                for (uint32_t w = unit0; ok && w < p.total_units; w += ustride) {
                    uint32_t t, sp, ukb0, ukb1;
                    unit_info(p, w, t, sp, ukb0, ukb1);
                    const uint32_t seg_kb = C_::SEG_KB ? C_::SEG_KB : (ukb1 - ukb0);
                    const uint32_t nseg = (ukb1 - ukb0 + seg_kb - 1) / seg_kb;
                    for (uint32_t sg = 0; ok && sg < nseg; sg++, u++) {
                        const uint32_t buf = u % NBUF, bph = (u / NBUF) & 1u;
                        if (!wait_bar(tempty_bar(buf), bph ^ 1u, abort_flag, p.status, DS_TIMEOUT_MMA,
                                      p.wait_limit_ns)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem_base + buf * BN;
                        const uint32_t kb0 = ukb0 + sg * seg_kb;
                        const uint32_t kb1 = min(ukb1, kb0 + seg_kb);
                        // Stages are taken p.mma_group at a time: wait for all of
                        // them, one fence, all their MMAs, then one commit each.
                        for (uint32_t kb = kb0; kb < kb1;) {
                            // at most STAGES: a group waits on distinct stages
                            const uint32_t grp = p.mma_group ? p.mma_group : C_::MMA_GROUP;
                            const uint32_t gn = min(min(grp, (uint32_t)STAGES), (kb1 - kb + KBS - 1) / KBS);
                            uint32_t st = stage, ph = phase;
                            for (uint32_t i = 0; i < gn; i++) {
                                if (!wait_bar(full_bar(st), ph, abort_flag, p.status, DS_TIMEOUT_MMA,
                                              p.wait_limit_ns)) {
                                    ok = false;
                                    break;
                                }
                                if (++st == STAGES) {
                                    st = 0;
                                    ph ^= 1u;
                                }
                            }
                            if (!ok) break;
                            tc_fence_after();
                            st = stage;
                            uint32_t kk = kb;                  // first k-block of stage st
                            for (uint32_t i = 0; i < gn; i++) {
                            const uint32_t nk = min((uint32_t)KBS, kb1 - kk);
#pragma unroll
                            for (uint32_t sub = 0; sub < (uint32_t)KBS; sub++) {
                            if (sub >= nk) break;
                            const uint32_t sA = sbase + st * C_::STAGE_BYTES + sub * C_::KB_BYTES;
                            const uint32_t sB = sA + C_::PLANES * C_::A_PLANE;
#pragma unroll
                            for (int j = 0; j < C_::KSTEPS; j++) {
                                uint64_t ad[C_::PLANES], bd[C_::PLANES];
#pragma unroll
                                for (int pl = 0; pl < C_::PLANES; pl++) {
                                    ad[pl] = A_MN ? smem_desc_sw128(sA + pl * C_::A_PLANE + j * C_::UK * ROW_BYTES,
                                                                    C_::SLAB, 1024)
                                                  : smem_desc_sw128(sA + pl * C_::A_PLANE + j * 32, 16, 1024);
                                    bd[pl] = B_MN ? smem_desc_sw128(sB + pl * C_::B_PLANE + j * C_::UK * ROW_BYTES,
                                                                    C_::SLAB, 1024)
                                                  : smem_desc_sw128(sB + pl * C_::B_PLANE + j * 32, 16, 1024);
                                }
                                const uint32_t first = (kk + sub == kb0 && j == 0) ? 0u : 1u;
                                if constexpr (KIND == K_TF32X3) {
                                    if constexpr (PAIR) {
                                        mma_tf32_pair(d, ad[1], bd[0], C_::IDESC, first);
                                        mma_tf32_pair(d, ad[0], bd[1], C_::IDESC, 1u);
                                        mma_tf32_pair(d, ad[0], bd[0], C_::IDESC, 1u);
                                    } else {
                                        mma_tf32(d, ad[1], bd[0], C_::IDESC, first);   // A_small * B_big
                                        mma_tf32(d, ad[0], bd[1], C_::IDESC, 1u);      // A_big * B_small
                                        mma_tf32(d, ad[0], bd[0], C_::IDESC, 1u);      // A_big * B_big
                                    }
                                } else {
                                    if constexpr (PAIR) mma_f16_pair(d, ad[0], bd[0], C_::IDESC, first);
                                    else mma_f16(d, ad[0], bd[0], C_::IDESC, first);
                                }
                            }
                            }
                            kk += nk;
                            if (++st == STAGES) st = 0;
                            }
                            for (uint32_t i = 0; i < gn; i++) {
                                if constexpr (PAIR) tc_commit_pair_mc(empty_bar(stage), 0x3);   // both CTAs' stage
                                else tc_commit(empty_bar(stage));
                                if (++stage == STAGES) {
                                    stage = 0;
                                    phase ^= 1u;
                                }
                            }
                            kb = kk;
                        }
                        if (!ok) break;
                        if constexpr (PAIR) tc_commit_pair_mc(tfull_bar(buf), 0x3);    // both epilogues
                        else tc_commit(tfull_bar(buf));
                    }
                }
                }
                // Never leave with MMAs in flight.
                if constexpr (PAIR) tc_commit_pair(drain_bar);
                else tc_commit(drain_bar);
                drain_bar_wait(drain_bar, 0, p.status, DS_TIMEOUT_MMA, DRAIN_LIMIT_NS);
            }
        }
    } else {
        if constexpr (C_::REG_SPLIT)
            asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C_::REGS_HIGH));
        // --------------------------------------------------------- epilogue
        // Launched as a programmatic dependent, this grid may start before the
        // previous kernel on the stream has finished: read alpha, beta and C
        // only after it has (as the TMA producer waits before its loads).
        if (!p.dep_end) asm volatile("griddepcontrol.wait;" ::: "memory");
        float alpha = p.alpha, beta = p.beta;
        load_scalars(p.d_alpha, p.d_beta, alpha, beta);
        const uint32_t q = (uint32_t)(warp & 3);          // TMEM lane quarter of this warp
        const uint32_t col0 = (uint32_t)((warp - C_::EPI_WARP0) / 4) * C_::EPI_COLS;   // this warp's columns
        const uint32_t row = q * 32u + (uint32_t)lane;
        const uint32_t lane_off = (q * 32u) << 16;
        // Only 2-byte small-M GEMMs run transposed; fp32 kernels leave that
        // store out, which keeps the segment sums in registers.
        constexpr bool IS_F32 = KIND == K_TF32X3;
        TOut* Cbase = reinterpret_cast<TOut*>(p.C);
        // This warp's two C staging boxes (EPI_STAGE) and the chunks staged so far.
        const uint32_t epi_box0 = epi_smem + (uint32_t)(warp - C_::EPI_WARP0) * 2u * C_::EPI_BOX;
        uint32_t kc = 0;
        uint32_t u = 0;                                       // accumulator hand-overs
        bool ok = true;
        // A split unit writes its fp32 partial tile to the workspace and no C;
        // split_reduce_kernel adds the splits in order and writes C.  Partial
        // tiles are stored column by column ([BN][BM], row fastest): lane =
        // row, so for each column a warp writes one contiguous 128-byte line.
        // Layout [split tile][split][half][BN][BM]: a pair tile has two
        // 128-row halves, one per CTA.
        auto split_publish = [&](uint32_t t, uint32_t sp, const float (&v)[32], int c) {
            const size_t half = ((size_t)(t - p.full_tiles) * p.split_s + sp) * (PAIR ? 2u : 1u) + rank;
            float* P = p.partial + half * BM * BN + (size_t)(col0 + c * 32) * BM + row;
#pragma unroll
            for (int i = 0; i < 32; i++) __stcg(P + i * BM, v[i]);
        };
        // Hand an accumulator buffer back to the MMA issuer.
        auto release = [&](uint32_t buf) {
            if constexpr (PAIR) mbar_arrive_cluster(to_issuer(tempty_bar(buf)));
            else mbar_arrive(tempty_bar(buf));
        };
        for (uint32_t w = unit0; ok && w < p.total_units; w += ustride) {
            uint32_t t, sp, ukb0, ukb1, b, mb, nb;
            unit_coords(p, w, t, sp, ukb0, ukb1, b, mb, nb);
            const uint32_t m = mb * C_::BM_TILE + rank * BM + row;
            TOut* cb = Cbase + p.sc * (int64_t)b;
            TOut* crow = cb + (size_t)m * p.ldc;
            if constexpr (C_::SEG_KB == 0) {
                const uint32_t buf = u % NBUF, bph = (u / NBUF) & 1u;
                ok = wait_bar(tfull_bar(buf), bph, abort_flag, p.status, DS_TIMEOUT_EPILOGUE,
                              p.wait_limit_ns);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
                if constexpr (C_::EPI_STAGE) {
                    if (sp == NO_SPLIT && p.c_tma) {
                        const int32_t mrow0 = (int32_t)(mb * C_::BM_TILE + rank * BM + q * 32u);
#pragma unroll 1
                        for (int c = 0; c < C_::EPI_COLS / 64; c++) {
                            uint32_t r[2][32];
                            const uint32_t ta = tmem_base + lane_off + buf * BN + col0 + c * 64;
                            tmem_ld_32x32b_x32(ta, r[0]);
                            tmem_ld_32x32b_x32(ta + 32, r[1]);
                            tmem_wait_ld();
                            const uint32_t n0 = nb * BN + col0 + c * 64;
                            if (n0 >= p.N || (uint32_t)mrow0 >= p.M) continue;      // warp-uniform
                            // Boxes alternate over the chunks stored: the store that read
                            // this box two stored chunks ago must be done with it.
                            const uint32_t box = epi_box0 + (kc++ & 1u) * C_::EPI_BOX;
                            if (lane == 0) bulk_wait_group_read<1>();
                            __syncwarp();
#pragma unroll
                            for (int g = 0; g < 8; g++) {
                                float old[8];
#pragma unroll
                                for (int i = 0; i < 8; i++) old[i] = 0.f;
                                const uint32_t n = n0 + g * 8;
                                if (beta != 0.f && m < p.M && n < p.N) {
                                    if (n + 8 <= p.N) {
                                        const uint4 o = *reinterpret_cast<const uint4*>(crow + n);
                                        const TOut* oh = reinterpret_cast<const TOut*>(&o);
#pragma unroll
                                        for (int i = 0; i < 8; i++) old[i] = Elem<TOut>::to_f(oh[i]);
                                    } else {
#pragma unroll
                                        for (int i = 0; i < 8; i++)
                                            if (n + i < p.N) old[i] = Elem<TOut>::to_f(crow[n + i]);
                                    }
                                }
                                uint4 out;
                                TOut* w8 = reinterpret_cast<TOut*>(&out);
#pragma unroll
                                for (int i = 0; i < 8; i++)
                                    w8[i] = Elem<TOut>::from_f(epilogue(
                                        alpha, __uint_as_float(r[g >> 2][(g & 3) * 8 + i]), beta, old[i]));
                                // SWIZZLE_128B: 16-byte chunk g of row `lane` sits at chunk g ^ (lane % 8).
                                st_shared_v4(box + (uint32_t)lane * ROW_BYTES + (((uint32_t)g ^ ((uint32_t)lane & 7u)) << 4), out);
                            }
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                const int32_t bz = (int32_t)b;
                                tma_store_3d(&p.tmC[0], box, (int32_t)n0, mrow0, bz);
                                for (uint32_t j = 0; j < p.npeers; j++)
                                    tma_store_3d(&p.tmC[1 + j], box, (int32_t)n0, mrow0, bz);
                                bulk_commit_group();
                            }
                        }
                        tc_fence_before();
                        release(buf);
                        u++;
                        continue;
                    }
                }
#pragma unroll 1
                for (int c = 0; c < C_::EPI_COLS / 32; c++) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tmem_base + lane_off + buf * BN + col0 + c * 32, r);
                    tmem_wait_ld();
                    const float(&v)[32] = reinterpret_cast<const float(&)[32]>(r);
                    if (sp != NO_SPLIT) {
                        split_publish(t, sp, v, c);
                    } else {
                        const uint32_t n0 = nb * BN + col0 + c * 32;
                        if (m < p.M && n0 < p.N) {
                            if (!IS_F32 && p.c_trans)
                                store_col32<TOut>(cb, m, n0, p.ldc, v, min(32u, p.N - n0), alpha, beta);
                            else
                                store_row32<TOut>(p, crow + n0, (size_t)(crow + n0 - Cbase), v,
                                                  min(32u, p.N - n0), p.c_vec_ok != 0, alpha, beta);
                        }
                    }
                }
                tc_fence_before();
                release(buf);
                u++;
            } else {
                // -0 is the exact identity of fp32 addition (-0 + x == x for
                // every x, -0 included): the first segment's sums come through
                // unchanged, and an unconditional add keeps them in registers.
                float sum[C_::EPI_COLS / 32][32];
#pragma unroll
                for (int c = 0; c < C_::EPI_COLS / 32; c++)
#pragma unroll
                    for (int i = 0; i < 32; i++) sum[c][i] = -0.f;
                const uint32_t nseg = (ukb1 - ukb0 + C_::SEG_KB - 1) / C_::SEG_KB;
                for (uint32_t sg = 0; sg < nseg; sg++, u++) {
                    const uint32_t buf = u % NBUF, bph = (u / NBUF) & 1u;
                    ok = wait_bar(tfull_bar(buf), bph, abort_flag, p.status, DS_TIMEOUT_EPILOGUE,
                                  p.wait_limit_ns);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < C_::EPI_COLS / 32; c++) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(tmem_base + lane_off + buf * BN + col0 + c * 32, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            sum[c][i] = __fadd_rn(sum[c][i], __uint_as_float(r[i]));
                    }
                    tc_fence_before();
                    release(buf);
                }
                if (!ok) break;
#pragma unroll
                for (int c = 0; c < C_::EPI_COLS / 32; c++) {
                    if (sp != NO_SPLIT) {
                        split_publish(t, sp, sum[c], c);
                    } else {
                        const uint32_t n0 = nb * BN + col0 + c * 32;
                        if (m < p.M && n0 < p.N) {
                            if (!IS_F32 && p.c_trans)
                                store_col32<TOut>(cb, m, n0, p.ldc, sum[c], min(32u, p.N - n0),
                                                  alpha, beta);
                            else
                                store_row32<TOut>(p, crow + n0, (size_t)(crow + n0 - Cbase),
                                                  sum[c], min(32u, p.N - n0), p.c_vec_ok != 0,
                                                  alpha, beta);
                        }
                    }
                }
            }
        }
        // Staged C boxes: every TMA store has written its data (and stopped
        // reading shared memory) before this CTA leaves.
        if constexpr (C_::EPI_STAGE)
            if (p.c_tma && lane == 0) bulk_wait_group_all();
        (void)epi_box0;
        (void)kc;
    }

    // Peer stores are made visible system-wide before the grid ends, so a
    // collective that follows on this stream (the replicas' rendezvous) orders them.
    if (p.npeers) __threadfence_system();
    __syncthreads();
    // A pair leaves together: the issuer's last commits arrive on the other
    // CTA's barriers, and its MMAs read the other CTA's shared memory.
    if constexpr (PAIR) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C_::TMEM_COLS);
        else tmem_dealloc(tmem_base, C_::TMEM_COLS);
    }
    // A grid that skipped the wait at its start ends after its prerequisite,
    // so work that depends on this grid also sees everything before it.
    if (p.dep_end && threadIdx.x == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Split tiles: C = alpha * (sum of the splits' partials in split order, fp32
// round-to-nearest) + beta * C.  One 32 x 8 block per 32-row x 64-column chunk:
// each thread issues the loads of up to four splits together (about S / 4
// round trips), the chunk is transposed through shared memory and written along C's
// rows.  Launched as a programmatic dependent of the GEMM grid that wrote the
// partials.
template <typename TOut, int BN, int TILE_ROWS>
__global__ void __launch_bounds__(256) split_reduce_kernel(const __grid_constant__ UmmaParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr uint32_t RC = 32, CC = 64;                // chunk rows x columns
    constexpr uint32_t CM = TILE_ROWS / RC, CN = BN / CC;
    constexpr uint32_t H = TILE_ROWS / BM;              // 128-row halves per tile
    __shared__ float tile[CC][RC + 1];                  // [column][row]
    const uint32_t st = blockIdx.x / (CM * CN);          // split tile
    const uint32_t r = blockIdx.x - st * (CM * CN);
    const uint32_t cm = r % CM, cn = r / CM;
    uint32_t b, mb, nb;
    tile_coords(p, p.full_tiles + st, b, mb, nb);
    float alpha = p.alpha, beta = p.beta;
    load_scalars(p.d_alpha, p.d_beta, alpha, beta);
    const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const uint32_t r0 = cm * RC;                        // chunk's first row in the tile
    const float* P = p.partial + ((size_t)st * p.split_s * H + r0 / BM) * BM * BN +
                     (size_t)(cn * CC + ty) * BM + (r0 % BM) + tx;
    const size_t qstride = (size_t)H * BM * BN;         // next split of the same half
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; j++) acc[j] = __ldcg(P + (size_t)j * 8 * BM);
    uint32_t q = 1;
    for (; q + 4 <= p.split_s; q += 4) {                // 32 loads in flight, added in order
        float x[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) x[i][j] = __ldcg(P + (size_t)(q + i) * qstride + (size_t)j * 8 * BM);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[j] = __fadd_rn(acc[j], x[i][j]);
    }
    for (; q < p.split_s; q++) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; j++) x[j] = __ldcg(P + (size_t)q * qstride + (size_t)j * 8 * BM);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = __fadd_rn(acc[j], x[j]);
    }
    TOut* const C0 = reinterpret_cast<TOut*>(p.C);
    TOut* C = C0 + p.sc * (int64_t)b;
    if (p.c_trans) {            // lanes run along C's rows already: store directly
        const uint32_t m = mb * TILE_ROWS + cm * RC + tx;
        if (m >= p.M) return;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t n = nb * BN + cn * CC + ty + 8 * j;
            if (n < p.N) {
                TOut* c = C + (size_t)n * p.ldc + m;
                const float old = beta != 0.f ? Elem<TOut>::to_f(*c) : 0.f;
                *c = Elem<TOut>::from_f(epilogue(alpha, acc[j], beta, old));
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) tile[ty + 8 * j][tx] = acc[j];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t rl = ty + 8 * j, m = mb * TILE_ROWS + cm * RC + rl;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t cl = h * 32 + tx, n = nb * BN + cn * CC + cl;
            if (m < p.M && n < p.N) {
                TOut* c = C + (size_t)m * p.ldc + n;
                const float old = beta != 0.f ? Elem<TOut>::to_f(*c) : 0.f;
                put_c(p, c, (size_t)(c - C0), Elem<TOut>::from_f(epilogue(alpha, tile[cl][rl], beta, old)));
            }
        }
    }
    if (p.npeers) __threadfence_system();
}

// 3xTF32 pre-pass: x -> big = rn_tf32(x), small = rn_tf32(x - big), written as
// compact [nb][rows][ldo] planes (ldo = cols rounded up to 4, pad columns zero).
__device__ __forceinline__ float rn_tf32(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7F800000u) == 0x7F800000u) return x;               // inf / nan unchanged
    u += 0xFFFu + ((u >> 13) & 1u);
    return __uint_as_float(u & 0xFFFFE000u);
}

// One operand's share of the pre-pass.  K-major (mn_major == 0): src[b][r][ld]
// with rows = M (or N) and cols = K, copied row by row.  MN-major: src[b][k][ld]
// with rows = K and cols = M (or N), written K-major (out[b][mn][ldo], K
// contiguous) so that the tf32 MMAs always read K-major operands.  Either way
// the output planes are [nb][MN][ldo] with ldo = K rounded up to 4 and the pad
// columns zero.  `blocks` CTAs of 256 threads work on it, striding over their
// work, so no grid dimension limits K or the batch count.
struct SplitJob {
    const float* src;
    uint32_t rows, cols, ld;
    int64_t bstride;
    uint32_t nb, ldo;
    float* big;
    float* small;
    uint32_t mn_major;
    uint32_t blocks;
};

__device__ __forceinline__ void split4(const float (&x)[4], float (&hi)[4], float (&lo)[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        hi[j] = rn_tf32(x[j]);
        lo[j] = isfinite(hi[j]) ? rn_tf32(x[j] - hi[j]) : 0.f;
    }
}

// K-major operand: 4 consecutive k per thread, 128-bit loads and stores.
__device__ __forceinline__ void split_rows(const SplitJob& j, uint32_t bid) {
    const uint32_t q = j.ldo / 4;
    const uint64_t total = (uint64_t)j.nb * j.rows * q;
    const bool vec_in = (j.ld & 3u) == 0 && (j.bstride & 3) == 0 &&
                        (reinterpret_cast<uintptr_t>(j.src) & 15u) == 0;
    for (uint64_t i = bid * 256ull + threadIdx.x; i < total; i += (uint64_t)j.blocks * 256u) {
        const uint64_t br = i / q;
        const uint32_t c0 = (uint32_t)(i - br * q) * 4u;
        const uint32_t b = (uint32_t)(br / j.rows), r = (uint32_t)(br - (uint64_t)b * j.rows);
        const float* s = j.src + j.bstride * (int64_t)b + (size_t)r * j.ld;
        float x[4], hi[4], lo[4];
        if (vec_in && c0 + 3 < j.cols) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(s + c0));
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
#pragma unroll
            for (int u = 0; u < 4; u++) x[u] = (c0 + u < j.cols) ? __ldg(s + c0 + u) : 0.f;
        }
        split4(x, hi, lo);
        const uint64_t o = br * j.ldo + c0;
        *reinterpret_cast<float4*>(j.big + o) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4*>(j.small + o) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// MN-major operand: 64 x 64 tiles transposed through shared memory; global
// reads (along MN) and writes (along K) are 128-bit when aligned.  The loop
// bound is the same for every thread of the block (the barriers need that).
constexpr int TT = 64;
__device__ __forceinline__ void split_cols(const SplitJob& j, uint32_t bid, float (*tile)[TT + 1]) {
    const uint32_t K = j.rows, MN = j.cols;
    const uint32_t tiles_mn = (MN + TT - 1) / TT, tiles_k = (j.ldo + TT - 1) / TT;
    const uint64_t total = (uint64_t)tiles_mn * tiles_k * j.nb;
    const uint32_t tx = threadIdx.x & 15, ty = threadIdx.x >> 4;    // 16 x 16
    const bool vec_in = (j.ld & 3u) == 0 && (j.bstride & 3) == 0 &&
                        (reinterpret_cast<uintptr_t>(j.src) & 15u) == 0;
    for (uint64_t t = bid; t < total; t += j.blocks) {
        const uint32_t mt = (uint32_t)(t % tiles_mn);
        const uint64_t rest = t / tiles_mn;
        const uint32_t kt = (uint32_t)(rest % tiles_k), b = (uint32_t)(rest / tiles_k);
        const uint32_t mn0 = mt * TT, k0 = kt * TT;
        const float* s = j.src + j.bstride * (int64_t)b;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t kl = ty + 16 * i, k = k0 + kl, mn = mn0 + tx * 4;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (k < K) {
                const float* row = s + (size_t)k * j.ld;
                if (vec_in && mn + 3 < MN) {
                    const float4 q = __ldg(reinterpret_cast<const float4*>(row + mn));
                    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
                } else {
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        if (mn + u < MN) v[u] = __ldg(row + mn + u);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++) tile[kl][tx * 4 + u] = v[u];
        }
        __syncthreads();
        const size_t obase = (size_t)b * MN * j.ldo;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t ml = ty + 16 * i, mn = mn0 + ml, k = k0 + tx * 4;
            if (mn < MN && k < j.ldo) {                  // ldo % 4 == 0: k..k+3 < ldo
                float x[4], hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; u++) x[u] = tile[tx * 4 + u][ml];
                split4(x, hi, lo);
                const size_t o = obase + (size_t)mn * j.ldo + k;
                *reinterpret_cast<float4*>(j.big + o) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(j.small + o) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        __syncthreads();
    }
}

// The whole pre-pass of a call in one launch: blocks [0, a.blocks) split A,
// the rest split B.
__global__ void __launch_bounds__(256) split_tf32_kernel(const SplitJob a, const SplitJob b) {
    __shared__ float tile[TT][TT + 1];                // [k][mn], MN-major jobs only
    const bool first = blockIdx.x < a.blocks;
    const uint32_t bid = first ? blockIdx.x : blockIdx.x - a.blocks;
    if (first) {
        if (a.mn_major) split_cols(a, bid, tile);
        else split_rows(a, bid);
    } else {
        if (b.mn_major) split_cols(b, bid, tile);
        else split_rows(b, bid);
    }
}

// ----------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        cudaGetLastError();
    });
    return fn;
}

// 3-D map over [nbatch][outer][inner] with element strides ld / bstride.
bool make_tmap(CUtensorMap* m, CUtensorMapDataType dt, uint32_t esize, const void* base,
               uint64_t inner, uint64_t outer, uint64_t ld, uint64_t nbatch, uint64_t bstride,
               uint32_t box_inner, uint32_t box_outer) {
    auto enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {inner, outer, nbatch};
    cuuint64_t strides[2] = {ld * esize, (nbatch > 1 ? bstride : outer * ld) * esize};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline uint32_t rup4(uint32_t x) { return (x + 3u) & ~3u; }

struct Operand {      // one operand as the tensor maps see it
    const void* base;
    uint64_t inner, outer, ld, nb, bstride;
    bool mn_major;
};

Operand operand_a(const GemmProblem& p) {
    Operand o;
    o.base = p.A;
    o.mn_major = p.op_a != 0;                       // A[k*lda + m]
    o.inner = o.mn_major ? p.M : p.K;
    o.outer = o.mn_major ? p.K : p.M;
    o.ld = p.lda;
    o.nb = (p.batch > 1 && p.sa != 0) ? p.batch : 1;
    o.bstride = (uint64_t)p.sa;
    return o;
}
Operand operand_b(const GemmProblem& p) {
    Operand o;
    o.base = p.B;
    o.mn_major = p.op_b == 0;                       // B[k*ldb + n]
    o.inner = o.mn_major ? p.N : p.K;
    o.outer = o.mn_major ? p.K : p.N;
    o.ld = p.ldb;
    o.nb = (p.batch > 1 && p.sb != 0) ? p.batch : 1;
    o.bstride = (uint64_t)p.sb;
    return o;
}

bool tma_ok_16bit(const Operand& o) {
    if (!al16(o.base) || (o.ld * 2) % 16 != 0 || o.ld < o.inner) return false;
    if (o.nb > 1 && ((o.bstride * 2) % 16 != 0 || o.bstride < o.outer * o.ld)) return false;
    return o.inner < (1ull << 32) && o.outer < (1ull << 31);
}

// 3xTF32 planes are always K-major: rows = the operand's M (or N), cols = K.
uint64_t plane_rows(const Operand& o) { return o.mn_major ? o.inner : o.outer; }
uint32_t plane_k(const Operand& o) { return (uint32_t)(o.mn_major ? o.outer : o.inner); }
uint64_t plane_elems(const Operand& o) { return o.nb * plane_rows(o) * rup4(plane_k(o)); }

// True when the registers a thread of this kernel is launched with, times its
// threads, cover the setmaxnreg split (warpgroup 0 at REGS_LOW, the rest at
// REGS_HIGH).  A split larger than that allocation would leave the epilogue
// warps' setmaxnreg.inc waiting forever, so such a kernel is never launched.
template <int KIND, bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR, int KBS = 1>
bool reg_split_fits() {
    using C_ = Cfg<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>;
    if constexpr (!C_::REG_SPLIT) {
        return true;
    } else {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, umma_gemm_kernel<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>) !=
            cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        const uint64_t have = (uint64_t)((fa.numRegs + 7) & ~7) * C_::THREADS;
        const uint64_t need = 128ull * C_::REGS_LOW + (uint64_t)(C_::THREADS - 128) * C_::REGS_HIGH;
        return fa.numRegs > 0 && have >= need;
    }
}

// One CTA per SM (persistent over `units` work units), or for PAIR one 2-CTA
// cluster per pair of SMs, as many clusters as the device can hold at once.
template <int KIND, bool A_MN, bool B_MN, int BN, int STAGES, bool PAIR, int KBS = 1>
cudaError_t launch_kind(const UmmaParams& prm, uint32_t units, int num_sms, cudaStream_t s,
                        bool pdl) {
    using C_ = Cfg<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>;
    auto kern = umma_gemm_kernel<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>;
    static std::atomic<uint64_t> attr_done{0};     // one bit per device
    static int max_clusters[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        if (!reg_split_fits<KIND, A_MN, B_MN, BN, STAGES, PAIR, KBS>()) return cudaErrorNotSupported;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C_::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (PAIR) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3((uint32_t)(num_sms & ~1));
            q.blockDim = dim3(C_::THREADS);
            q.dynamicSmemBytes = C_::SMEM_BYTES;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
            q.attrs = at;
            q.numAttrs = 1;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, kern, &q);
            if (e != cudaSuccess || n < 1) {
                cudaGetLastError();
                return cudaErrorNotSupported;
            }
            max_clusters[dev & 63] = n;
            if (getenv("VKBLAS_TRACE"))
                fprintf(stderr, "[vkblas] device %d: %d resident 2-CTA clusters for %s, %d-wide tiles (%d SMs)\n",
                        dev, n, KIND == K_TF32X3 ? "3xTF32" : "kind::f16", BN, num_sms);
        }
        attr_done.fetch_or(bit);
    }
    // pdl: launched as the programmatic dependent of the kernel before it on
    // the stream (the 3xTF32 pre-pass); see griddepcontrol.wait in the kernel.
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(C_::THREADS);
    cfg.dynamicSmemBytes = C_::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    unsigned n_at = 0;
    if (PAIR) {
        const uint32_t mc = (uint32_t)max_clusters[dev & 63];
        cfg.gridDim = dim3(2 * (units < mc ? units : mc));
        at[n_at].id = cudaLaunchAttributeClusterDimension;
        at[n_at].val.clusterDim.x = 2; at[n_at].val.clusterDim.y = 1; at[n_at].val.clusterDim.z = 1;
        n_at++;
    } else {
        cfg.gridDim = dim3(units < (uint32_t)num_sms ? units : (uint32_t)num_sms);
    }
    if (pdl) {
        at[n_at].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n_at].val.programmaticStreamSerializationAllowed = 1;
        n_at++;
    }
    cfg.attrs = at;
    cfg.numAttrs = n_at;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm);
    count_launch();
    return e;
}

// 2-byte GEMMs are launched as programmatic dependents of whatever kernel
// precedes them on the stream (VKBLAS_PDL=0: plain launches).  Their CTAs
// may then take SMs the previous grid has left and run their prologue
// (barriers, TMEM, tensor maps) early; every global access waits in
// griddepcontrol.wait until the previous grid has finished.
bool pdl_all() {
    static const bool on = [] {
        const char* e = getenv("VKBLAS_PDL");
        return !(e && *e && atoi(e) == 0);
    }();
    return on;
}

template <int KIND, int BN, int STAGES, bool PAIR, int KBS = 1>
cudaError_t launch_majors(bool a_mn, bool b_mn, const UmmaParams& prm, uint32_t units, int num_sms,
                          cudaStream_t s) {
    const bool pdl = pdl_all();
    if (!a_mn && !b_mn) return launch_kind<KIND, false, false, BN, STAGES, PAIR, KBS>(prm, units, num_sms, s, pdl);
    if (!a_mn && b_mn) return launch_kind<KIND, false, true, BN, STAGES, PAIR, KBS>(prm, units, num_sms, s, pdl);
    if (a_mn && !b_mn) return launch_kind<KIND, true, false, BN, STAGES, PAIR, KBS>(prm, units, num_sms, s, pdl);
    return launch_kind<KIND, true, true, BN, STAGES, PAIR, KBS>(prm, units, num_sms, s, pdl);
}

// The reduce of split tiles, launched so that it may become resident while
// the GEMM grid drains (programmatic stream serialization).
template <typename TOut, int BN, int TILE_ROWS = BM>
cudaError_t launch_reduce(const UmmaParams& prm, cudaStream_t s) {
    const uint32_t chunks = (prm.total_tiles - prm.full_tiles) * (TILE_ROWS / 32) * (BN / 64);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(chunks);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, split_reduce_kernel<TOut, BN, TILE_ROWS>, prm);
    count_launch();
    return e;
}

constexpr int BN_16 = 256, STAGES_16 = 4;
constexpr int BN_TF32 = 128, STAGES_TF32 = 3;
// CTA pairs (256-row tiles): half of B per CTA leaves room for deeper rings.
constexpr int STAGES_16P = 6, STAGES_TF32P = 4;
// fp16 / bf16 pairs with two k-blocks per stage: three 64 KB stages.
constexpr int STAGES_16P2 = 3;
// Narrow tail of fp16 / bf16 pair grids: 256 x 128 tiles, four 48 KB stages of
// two k-blocks each.
constexpr int BN_16T = 128, STAGES_16T = 4;
// 3xTF32 on CTA pairs with 256 x 256 tiles: 64 KB stages (big and small
// planes of 128 A rows and 128 B rows per CTA).
constexpr int BN_TF32W = 256, STAGES_TF32W = 3;

// Stages the MMA issuer takes at a time: VKBLAS_MMA_GROUP=1-4 sets it for
// every kernel, unset (0) leaves each kernel's own (Cfg::MMA_GROUP).
uint32_t mma_group() {
    static const uint32_t g = [] {
        const char* e = getenv("VKBLAS_MMA_GROUP");
        const int v = e ? atoi(e) : 0;
        return (uint32_t)(v < 0 ? 0 : v > 4 ? 4 : v);
    }();
    return g;
}

// k-blocks per stage of the fp16 / bf16 pair kernel: VKBLAS_F16_KBS=1 keeps
// six one-k-block stages (with the issuer taking two at a time), else two
// k-blocks per stage.
// k-blocks per stage of the small-M (transposed) kernel: 2 (four 48 KB
// stages) unless VKBLAS_SM_KBS says 1 (eight 24 KB stages) or 4 (two 96 KB).
// Measured on B200 (4096 -> 14336, graph replay), 1 / 2 / 4: M = 16 32.8 /
// 23.4 / 25.3 us, M = 32 33.2 / 23.9 / 25.7 us, M = 64 34.5 / 25.3 / 27.2 us.
int small_m_kbs() {
    static const int k = [] {
        const char* e = getenv("VKBLAS_SM_KBS");
        const int v = e && *e ? atoi(e) : 2;
        return v == 1 || v == 4 ? v : 2;
    }();
    return k;
}

int f16_pair_kbs() {
    static const int k = [] {
        const char* e = getenv("VKBLAS_F16_KBS");
        return (e && *e && atoi(e) == 1) ? 1 : 2;
    }();
    return k;
}

// Tile order: groups of M-blocks sweep the N-blocks together, so that the
// tiles running at the same time share A rows and B columns in L2.
// VKBLAS_GROUP_M=n fixes the group size; 0 (unset) lets launch_umma_gemm pick.
uint32_t group_m() {
    static const uint32_t g = [] {
        const char* e = getenv("VKBLAS_GROUP_M");
        const int v = e && *e ? atoi(e) : 0;
        return (uint32_t)(v < 0 ? 0 : v > 64 ? 64 : v);
    }();
    return g;
}

// VKBLAS_EPI_TMA=0 keeps the 2-byte epilogues on direct global stores.
bool epi_tma_enabled() {
    static const bool on = [] {
        const char* e = getenv("VKBLAS_EPI_TMA");
        return !(e && *e && atoi(e) == 0);
    }();
    return on;
}

// VKBLAS_TC_PAIR=0 keeps every tensor-core GEMM on single-CTA tiles.
bool pair_enabled() {
    static const bool on = [] {
        const char* e = getenv("VKBLAS_TC_PAIR");
        return !(e && *e && atoi(e) == 0);
    }();
    return on;
}

// 3xTF32 GEMMs on CTA pairs with N >= 256 use 256-wide tiles: each MMA
// computes twice the columns for the same A tile, which halves the A operand's
// shared-memory reads and the MMA count per flop (measured on B200 at 4096^3:
// the GEMM kernel 0.577 -> 0.465 ms).  VKBLAS_TF32_WIDE=0 keeps 128-wide
// tiles.  Taken only when the kernel's register split fits.
bool tf32_wide() {
    static const bool on = [] {
        const char* e = getenv("VKBLAS_TF32_WIDE");
        return !(e && *e && atoi(e) == 0) &&
               reg_split_fits<K_TF32X3, false, false, BN_TF32W, STAGES_TF32W, true>();
    }();
    return on;
}
// Small-M 2-byte GEMMs (decode with up to 64 tokens) run transposed: weight
// rows on the MMA's 128 lanes, tokens on a 64-wide N tile, an 8-deep ring.
constexpr int BN_SM = 64, STAGES_SM = 8;
constexpr uint32_t K_ROT_MUL = 29;
constexpr uint32_t SMALL_M_MAX = 64;

bool small_m_swap(const GemmProblem& p) {
    return (p.dtype == DT_F16 || p.dtype == DT_BF16) && p.M <= SMALL_M_MAX && p.N >= 128;
}

// C^T = op(B)^T op(A)^T in the engine's row-major terms: op(B)^T is B read
// with the opposite transpose flag, and likewise for A.
GemmProblem swapped(const GemmProblem& p) {
    GemmProblem q = p;
    q.M = p.N;
    q.N = p.M;
    q.A = p.B; q.lda = p.ldb; q.sa = p.sb; q.op_a = p.op_b ? 0 : 1;
    q.B = p.A; q.ldb = p.lda; q.sb = p.sa; q.op_b = p.op_a ? 0 : 1;
    return q;
}

// The problem the kernel runs, its tile and whether CTA pairs run it (256-row
// tiles whenever M fills them).
struct KernelShape {
    GemmProblem q;
    bool c_trans;
    uint32_t BN;
    bool pair;
    uint32_t bm_tile;
};
// `wide`: whether 256-wide 3xTF32 pair tiles may be chosen (tf32_wide() on the
// launch path).
KernelShape kernel_shape(const GemmProblem& p, bool wide) {
    if (small_m_swap(p)) return {swapped(p), true, (uint32_t)BN_SM, false, (uint32_t)BM};
    const bool pair = pair_enabled() && p.M >= 2u * BM;
    uint32_t bn = p.dtype == DT_F32 ? (uint32_t)BN_TF32 : (uint32_t)BN_16;
    if (p.dtype == DT_F32 && pair && p.N >= (uint32_t)BN_TF32W && wide) bn = BN_TF32W;
    return {p, false, bn, pair, (uint32_t)(pair ? 2 * BM : BM)};
}
KernelShape kernel_shape(const GemmProblem& p) { return kernel_shape(p, tf32_wide()); }

// Work decomposition.  Whole waves of tiles run unsplit; the tiles of the
// last, partial wave (all tiles when there are fewer tiles than SMs -- the
// reference's skinny split-K case, src/vkblas.c:2850-2867) are cut along K
// into S ranges so that the last wave fills the GPU, when that saves more
// than the split costs: the partial tiles make a round trip through L2 and a
// second kernel adds them (measured on B200: about 10 us for a wave of
// 128 x 256 tiles), so at least MIN_SAVED_KB k-blocks of a tile's MMA time
// (about 0.37 us each for fp16, 0.7 us for 3xTF32) must go.
struct SplitPlan {
    uint32_t full, s, kb_per, units;
    size_t partial_bytes;
    uint32_t tail;       // last-wave tiles run as 256 x 128 halves in a second grid
};

// VKBLAS_NARROW_TAIL=0 keeps the last wave of fp16 / bf16 pair tiles whole.
bool narrow_tail_enabled() {
    static const bool on = [] {
        const char* e = getenv("VKBLAS_NARROW_TAIL");
        return !(e && *e && atoi(e) == 0);
    }();
    return on;
}

SplitPlan plan_split(const KernelShape& ks, int num_sms) {
    const GemmProblem& p = ks.q;
    const bool is32 = p.dtype == DT_F32;
    const uint32_t BN = ks.BN;
    const uint32_t BK = ROW_BYTES / (is32 ? 4u : 2u);
    const uint32_t seg = is32 ? 8u : 1u;                // 3xTF32 accumulates 8-k-block segments
    // 128 x 64 small-M tiles stream weights (~0.3 us per k-block) and their
    // partial tiles are a quarter of a 128 x 256 tile's.
    const uint32_t min_saved_kb = is32 ? 16u : (BN == (uint32_t)BN_SM ? 8u : 48u);
    const uint64_t T =
        (uint64_t)((p.M + ks.bm_tile - 1) / ks.bm_tile) * ((p.N + BN - 1) / BN) * p.batch;
    const uint32_t num_kb = (p.K + BK - 1) / BK;
    SplitPlan pl{(uint32_t)T, 1, num_kb, (uint32_t)T, 0, 0};
    // Workers: SMs, or SM pairs for 256-row tiles (the per-SM work of a tile
    // and its k-block time are the same in both cases).
    const int workers = ks.pair ? num_sms / 2 : num_sms;
    const uint64_t P = (uint64_t)(workers > 0 ? workers : 1);
    const uint64_t rem = T % P;
    if (rem == 0 || T >= (1ull << 31)) return pl;
    uint32_t S = (uint32_t)(P / rem);
    if (S > 16) S = 16;
    const uint32_t min_kb = seg > 4 ? seg : 4;
    if (S > num_kb / min_kb) S = num_kb / min_kb;
    if (S < 2) return pl;
    uint32_t kb_per = (num_kb + S - 1) / S;
    kb_per = (kb_per + seg - 1) / seg * seg;
    const uint32_t s2 = (num_kb + kb_per - 1) / kb_per;
    if (s2 < 2 || num_kb - kb_per < min_saved_kb) return pl;
    // Where the last wave would be split along K, 2-byte 256 x 256 pair tiles
    // of a long grid (8 waves or more) whose last wave fills at most half of
    // the SM pairs run as twice as many 256 x 128 halves instead, in one wave
    // of a second grid, with no partial sums to write and add.  A half tile
    // reads its A rows again, so it pays only where the tail is a small part
    // of the work.  Measured on B200 against the split: 16384^3 (26 of 4096
    // tiles) 6149 -> 5998 and 6156 -> 6048 us; 4096 x 4096 x 16384 (34 of
    // 256) 387 -> 401 us.  Without a split neither pays: 4096^3 101.4 -> 106.1 us.
    if (!is32 && ks.pair && !ks.c_trans && BN == 256u && T >= 8 * P && 2 * rem <= P &&
        narrow_tail_enabled()) {
        pl.full = pl.units = (uint32_t)(T - rem);
        pl.tail = (uint32_t)rem;
        return pl;
    }
    pl.full = (uint32_t)(T - rem);
    pl.s = s2;
    pl.kb_per = kb_per;
    pl.units = pl.full + (uint32_t)rem * s2;
    pl.partial_bytes = (size_t)rem * s2 * ks.bm_tile * BN * sizeof(float);
    return pl;
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* m, bool bf16, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t ld, uint32_t box_inner, uint32_t box_outer) {
    auto enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
               const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool umma_supported(const GemmProblem& p) {
    if (!encode_fn()) return false;
    if (p.dtype == DT_F16 || p.dtype == DT_BF16)
        return tma_ok_16bit(operand_a(p)) && tma_ok_16bit(operand_b(p));
    if (p.dtype == DT_F32) {
        Operand a = operand_a(p), b = operand_b(p);
        return a.inner < (1ull << 31) && a.outer < (1ull << 21) * 32 && b.inner < (1ull << 31) &&
               b.outer < (1ull << 21) * 32;
    }
    return false;
}

bool umma_profitable(const GemmProblem& p) {
    if ((uint64_t)p.M * p.N * p.K < (1ull << 21)) return false;
    return (p.M >= 32 && p.N >= 32) || small_m_swap(p);
}

bool umma_uses_pair(const GemmProblem& p, int num_sms, bool split_ws) {
    (void)num_sms;
    (void)split_ws;
    return kernel_shape(p).pair;
}

int umma_tile_n(const GemmProblem& p) { return (int)kernel_shape(p).BN; }

UmmaPlan umma_plan(const GemmProblem& p, int num_sms, bool allow_wide) {
    const KernelShape ks = kernel_shape(p, allow_wide);
    const SplitPlan pl = plan_split(ks, num_sms);
    const GemmProblem& q = ks.q;
    const uint32_t bk = ROW_BYTES / (q.dtype == DT_F32 ? 4u : 2u);
    UmmaPlan r;
    r.tile_m = ks.bm_tile;
    r.tile_n = ks.BN;
    r.transposed = ks.c_trans ? 1u : 0u;
    r.pair = ks.pair ? 1u : 0u;
    r.tiles = (pl.s > 1 ? pl.full + (pl.units - pl.full) / pl.s : pl.units) + pl.tail;
    r.full_tiles = pl.full;
    r.tail_tiles = pl.tail;
    r.splits = pl.s;
    r.kblocks = (q.K + bk - 1) / bk;
    r.kblocks_per_split = pl.kb_per;
    r.partial_bytes = pl.s > 1 ? (uint64_t)pl.partial_bytes : 0u;
    r.too_many_tiles = (uint64_t)((q.M + ks.bm_tile - 1) / ks.bm_tile) * ((q.N + ks.BN - 1) / ks.BN) *
                           q.batch >= (1ull << 31);
    return r;
}

int umma_split_count(const GemmProblem& p, int num_sms) {
    return (int)plan_split(kernel_shape(p), num_sms).s;
}

size_t umma_split_workspace_bytes(const GemmProblem& p, int num_sms) {
    const SplitPlan pl = plan_split(kernel_shape(p), num_sms);
    return pl.s > 1 ? pl.partial_bytes : 0;
}

size_t umma_workspace_bytes(const GemmProblem& p) {
    if (p.dtype != DT_F32) return 0;
    const uint64_t a = plane_elems(operand_a(p)), b = plane_elems(operand_b(p));
    // big and small planes of A and B, each 256-byte aligned
    return (size_t)(2 * ((a * 4 + 255) / 256 * 256) + 2 * ((b * 4 + 255) / 256 * 256));
}

cudaError_t launch_umma_gemm(const GemmProblem& p_in, int num_sms, int* d_status, void* ws,
                             void* split_ws, bool test_stall, cudaStream_t s, cudaEvent_t ev_start,
                             cudaEvent_t ev_end, void* const* peers, uint32_t npeers) {
    // Peer copies: at most 7, none null; the transposed small-M epilogue
    // (column stores) does not write them.
    if (npeers > 7 || (npeers && !peers)) return cudaErrorInvalidValue;
    for (uint32_t j = 0; j < npeers; j++)
        if (!peers[j]) return cudaErrorInvalidValue;
    if (npeers && small_m_swap(p_in)) return cudaErrorNotSupported;
    UmmaParams prm;
    memset(&prm, 0, sizeof(prm));
    prm.tail_first = NO_TAIL;
    for (uint32_t j = 0; j < npeers; j++) prm.peer[j] = peers[j];
    prm.npeers = npeers;
    prm.wait_limit_ns = test_stall ? TEST_WAIT_LIMIT_NS : WAIT_LIMIT_NS;
    prm.mma_group = mma_group();
    prm.test_skip_first_load = test_stall ? 1u : 0u;
    const KernelShape ks = kernel_shape(p_in);
    const GemmProblem& p = ks.q;                 // the (possibly transposed) problem run
    prm.c_trans = ks.c_trans ? 1u : 0u;
    // Rotated k order for the weight-streaming tiles.  Measured on B200 at
    // 4096 -> 14336, M = 16-64: multiplier 29 took 24.9-26.7 us to
    // 23.5-25.3 us; 7 gained less; 1 (neighbouring tiles one k-block apart)
    // lost 1 us.  Large tiles keep the plain order, because neighbouring
    // tiles there share A and B k-blocks in L2.
    prm.k_rot_mul = ks.c_trans ? K_ROT_MUL : 0u;
    const Operand a = operand_a(p), b = operand_b(p);
    const bool is32 = p.dtype == DT_F32;
    const int BN = (int)ks.BN;
    const uint32_t esize = is32 ? 4u : 2u;
    const uint32_t BK = ROW_BYTES / esize, EPB = ROW_BYTES / esize;
    // 256-row tiles on CTA pairs when no split is planned and M fills them.
    const SplitPlan pl = plan_split(ks, num_sms);
    const bool pair = ks.pair;
    bool pdl = false;                           // the GEMM follows the 3xTF32 pre-pass
    const uint32_t bn_cta = pair ? (uint32_t)BN / 2 : (uint32_t)BN;      // B rows per CTA

    auto box_for = [&](const Operand& o, uint32_t tile_rows, uint32_t& bi, uint32_t& bo) {
        if (o.mn_major) { bi = EPB; bo = BK; }          // 128-byte MN slab x BK k-rows
        else { bi = BK; bo = tile_rows; }               // BK k (128 bytes) x tile rows
    };
    uint32_t abi, abo, bbi, bbo;
    box_for(a, BM, abi, abo);
    box_for(b, bn_cta, bbi, bbo);

    if (!is32) {
        const CUtensorMapDataType dt =
            p.dtype == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        if (!make_tmap(&prm.tmA[0], dt, 2, a.base, a.inner, a.outer, a.ld, a.nb, a.bstride, abi, abo) ||
            !make_tmap(&prm.tmB[0], dt, 2, b.base, b.inner, b.outer, b.ld, b.nb, b.bstride, bbi, bbo))
            return cudaErrorNotSupported;
    } else {
        if (!ws) return cudaErrorNotSupported;
        const uint64_t ae = plane_elems(a), be = plane_elems(b);
        char* w = reinterpret_cast<char*>(ws);
        float* a_big = reinterpret_cast<float*>(w);
        w += (ae * 4 + 255) / 256 * 256;
        float* a_small = reinterpret_cast<float*>(w);
        w += (ae * 4 + 255) / 256 * 256;
        float* b_big = reinterpret_cast<float*>(w);
        w += (be * 4 + 255) / 256 * 256;
        float* b_small = reinterpret_cast<float*>(w);
        const uint32_t lda_o = rup4(plane_k(a)), ldb_o = rup4(plane_k(b));
        const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const uint64_t ar = plane_rows(a), br = plane_rows(b);
        const uint64_t sa_o = ar * lda_o, sb_o = br * ldb_o;
        // K-major boxes: BK (32 fp32 = 128 bytes) x tile rows
        if (!make_tmap(&prm.tmA[0], dt, 4, a_big, plane_k(a), ar, lda_o, a.nb, sa_o, BK, BM) ||
            !make_tmap(&prm.tmA[1], dt, 4, a_small, plane_k(a), ar, lda_o, a.nb, sa_o, BK, BM) ||
            !make_tmap(&prm.tmB[0], dt, 4, b_big, plane_k(b), br, ldb_o, b.nb, sb_o, BK, bn_cta) ||
            !make_tmap(&prm.tmB[1], dt, 4, b_small, plane_k(b), br, ldb_o, b.nb, sb_o, BK, bn_cta))
            return cudaErrorNotSupported;
        // One launch splits both operands; the GEMM below is its programmatic
        // dependent (its producer waits in griddepcontrol.wait before the first
        // load of a plane), so the GEMM's launch and set-up overlap the
        // pre-pass's last blocks.
        auto job = [&](const Operand& o, uint32_t ldo, float* big, float* small) {
            SplitJob j;
            j.src = reinterpret_cast<const float*>(o.base);
            j.rows = (uint32_t)o.outer;
            j.cols = (uint32_t)o.inner;
            j.ld = (uint32_t)o.ld;
            j.bstride = (int64_t)o.bstride;
            j.nb = (uint32_t)o.nb;
            j.ldo = ldo;
            j.big = big;
            j.small = small;
            j.mn_major = o.mn_major ? 1u : 0u;
            // about 16 blocks of work per SM, each striding over the rest
            const uint64_t work = o.mn_major
                ? (uint64_t)((o.inner + TT - 1) / TT) * ((ldo + TT - 1) / TT) * o.nb
                : (o.nb * o.outer * (ldo / 4) + 255) / 256;
            const uint64_t cap = (uint64_t)num_sms * 16;
            j.blocks = (uint32_t)(work < 1 ? 1 : work < cap ? work : cap);
            return j;
        };
        const SplitJob ja = job(a, lda_o, a_big, a_small), jb = job(b, ldb_o, b_big, b_small);
        split_tf32_kernel<<<ja.blocks + jb.blocks, 256, 0, s>>>(ja, jb);
        count_launch();
        pdl = true;
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    prm.C = p.C;
    prm.ldc = p.ldc;
    prm.sc = p.sc;
    prm.M = p.M; prm.N = p.N; prm.K = p.K; prm.batch = p.batch;
    const uint32_t bm_tile = ks.bm_tile;
    prm.tiles_m = (p.M + bm_tile - 1) / bm_tile;
    prm.tiles_n = (p.N + BN - 1) / BN;
    // Tile order.  Measured on B200 (one box), group of 8 -> all 16 M-blocks:
    // HGEMM 4096^3 102.0 -> 100.3 us, but 3xTF32 SGEMM 4096^3 539.9 -> 543.7 us,
    // and at 8192^3 (32 M-blocks) groups of 16 / 32 lost 2% / 10%.
    prm.group_m = group_m() ? group_m() : (!is32 && prm.tiles_m <= 16u) ? 16u : 8u;
    prm.num_kb = (p.K + BK - 1) / BK;
    const uint64_t total = (uint64_t)prm.tiles_m * prm.tiles_n * p.batch;
    if (total >= (1ull << 31)) return cudaErrorNotSupported;
    prm.total_tiles = (uint32_t)total;
    if (pl.s > 1 && split_ws) {
        prm.full_tiles = pl.full;
        prm.split_s = pl.s;
        prm.split_kb = pl.kb_per;
        prm.total_units = pl.units;
        prm.partial = reinterpret_cast<float*>(split_ws);
    } else {
        prm.full_tiles = prm.total_tiles;
        prm.split_s = 1;
        prm.split_kb = prm.num_kb;
        prm.total_units = prm.total_tiles;
    }
    // C stored from shared memory by TMA (kernels with Cfg::EPI_STAGE): C and
    // every peer copy 16-byte aligned, rows of whole 16-byte units that do
    // not overlap, batch entries likewise, and N a multiple of 8.  Measured
    // on B200: a TMA store clipped at an N that ends inside a 16-byte unit
    // still wrote the rest of that unit (the ldc padding after column N).
    if (!is32 && !ks.c_trans && epi_tma_enabled()) {
        const CUtensorMapDataType dt =
            p.dtype == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        const uint64_t nbc = p.batch > 1 ? p.batch : 1;
        bool okc = al16(p.C) && ((uint64_t)p.ldc * 2) % 16 == 0 && p.ldc >= p.N && p.N % 8 == 0 &&
                   (nbc == 1 || (((uint64_t)p.sc * 2) % 16 == 0 &&
                                 (uint64_t)p.sc >= (uint64_t)p.M * p.ldc));
        for (uint32_t j = 0; okc && j < npeers; j++) okc = al16(peers[j]);
        okc = okc && make_tmap(&prm.tmC[0], dt, 2, p.C, p.N, p.M, p.ldc, nbc, (uint64_t)p.sc, 64, 32);
        for (uint32_t j = 0; okc && j < npeers; j++)
            okc = make_tmap(&prm.tmC[1 + j], dt, 2, peers[j], p.N, p.M, p.ldc, nbc, (uint64_t)p.sc, 64, 32);
        prm.c_tma = okc ? 1u : 0u;
    }
    prm.a_batched = a.nb > 1;
    prm.b_batched = b.nb > 1;
    prm.alpha = p.alpha; prm.beta = p.beta; prm.d_alpha = p.d_alpha; prm.d_beta = p.d_beta;
    prm.status = d_status;
    prm.c_vec_ok = al16(p.C) && ((uint64_t)p.ldc * esize) % 16 == 0 &&
                   (p.batch == 1 || ((uint64_t)p.sc * esize) % 16 == 0);
    // Narrow tail: this grid runs the whole tiles; a second grid, launched
    // right after it as its programmatic dependent, runs the last wave's
    // pl.tail tiles as 256 x 128 halves.  Its B tensor map has 64-row boxes.
    UmmaParams prmT;
    if (pl.tail) {
        prm.full_tiles = prm.total_units = prm.total_tiles - pl.tail;
        prmT = prm;
        prmT.tail_first = prm.total_tiles - pl.tail;
        prmT.full_tiles = prmT.total_units = 2 * pl.tail;
        prmT.dep_end = 1;
        uint32_t tbi, tbo;
        box_for(b, BN_16T / 2, tbi, tbo);
        const CUtensorMapDataType dt =
            p.dtype == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        if (!make_tmap(&prmT.tmB[0], dt, 2, b.base, b.inner, b.outer, b.ld, b.nb, b.bstride, tbi, tbo))
            return cudaErrorNotSupported;
    }
    const uint32_t units = prm.total_units;
    const bool amn = a.mn_major, bmn = b.mn_major;
    cudaError_t e;
    const bool sm = ks.c_trans;
    if (ev_start) cudaEventRecord(ev_start, s);        // after the 3xTF32 pre-pass
    switch (p.dtype) {
        case DT_F16:
            e = sm     ? (small_m_kbs() == 2 ? launch_majors<K_F16, BN_SM, STAGES_SM / 2, false, 2>(amn, bmn, prm, units, num_sms, s)
                          : small_m_kbs() == 4 ? launch_majors<K_F16, BN_SM, STAGES_SM / 4, false, 4>(amn, bmn, prm, units, num_sms, s)
                                               : launch_majors<K_F16, BN_SM, STAGES_SM, false>(amn, bmn, prm, units, num_sms, s))
                : (pair && f16_pair_kbs() == 2)
                    ? launch_majors<K_F16, BN_16, STAGES_16P2, true, 2>(amn, bmn, prm, units, num_sms, s)
                : pair ? launch_majors<K_F16, BN_16, STAGES_16P, true>(amn, bmn, prm, units, num_sms, s)
                       : launch_majors<K_F16, BN_16, STAGES_16, false>(amn, bmn, prm, units, num_sms, s);
            break;
        case DT_BF16:
            e = sm     ? (small_m_kbs() == 2 ? launch_majors<K_BF16, BN_SM, STAGES_SM / 2, false, 2>(amn, bmn, prm, units, num_sms, s)
                          : small_m_kbs() == 4 ? launch_majors<K_BF16, BN_SM, STAGES_SM / 4, false, 4>(amn, bmn, prm, units, num_sms, s)
                                               : launch_majors<K_BF16, BN_SM, STAGES_SM, false>(amn, bmn, prm, units, num_sms, s))
                : (pair && f16_pair_kbs() == 2)
                    ? launch_majors<K_BF16, BN_16, STAGES_16P2, true, 2>(amn, bmn, prm, units, num_sms, s)
                : pair ? launch_majors<K_BF16, BN_16, STAGES_16P, true>(amn, bmn, prm, units, num_sms, s)
                       : launch_majors<K_BF16, BN_16, STAGES_16, false>(amn, bmn, prm, units, num_sms, s);
            break;
        case DT_F32:   // planes are K-major whatever op(A), op(B) are
            e = !pair ? launch_kind<K_TF32X3, false, false, BN_TF32, STAGES_TF32, false>(prm, units, num_sms, s, pdl)
                : BN == BN_TF32W
                    ? launch_kind<K_TF32X3, false, false, BN_TF32W, STAGES_TF32W, true>(prm, units, num_sms, s, pdl)
                    : launch_kind<K_TF32X3, false, false, BN_TF32, STAGES_TF32P, true>(prm, units, num_sms, s, pdl);
            break;
        default: return cudaErrorInvalidValue;
    }
    if (e == cudaSuccess && pl.tail) {
        const uint32_t tu = prmT.total_units;
        e = p.dtype == DT_F16
                ? launch_majors<K_F16, BN_16T, STAGES_16T, true, 2>(amn, bmn, prmT, tu, num_sms, s)
                : launch_majors<K_BF16, BN_16T, STAGES_16T, true, 2>(amn, bmn, prmT, tu, num_sms, s);
    }
    if (e == cudaSuccess && prm.split_s > 1) {
        switch (p.dtype) {
            case DT_F16:
                e = sm     ? launch_reduce<__half, BN_SM>(prm, s)
                    : pair ? launch_reduce<__half, BN_16, 2 * BM>(prm, s)
                           : launch_reduce<__half, BN_16>(prm, s);
                break;
            case DT_BF16:
                e = sm     ? launch_reduce<__nv_bfloat16, BN_SM>(prm, s)
                    : pair ? launch_reduce<__nv_bfloat16, BN_16, 2 * BM>(prm, s)
                           : launch_reduce<__nv_bfloat16, BN_16>(prm, s);
                break;
            default:
                e = !pair ? launch_reduce<float, BN_TF32>(prm, s)
                    : BN == BN_TF32W ? launch_reduce<float, BN_TF32W, 2 * BM>(prm, s)
                                     : launch_reduce<float, BN_TF32, 2 * BM>(prm, s);
        }
    }
    if (ev_end && e == cudaSuccess) cudaEventRecord(ev_end, s);
    return e;
}

}  // namespace vkb
