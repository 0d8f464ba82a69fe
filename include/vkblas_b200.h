/* vkblas_b200.h -- B200-specific extensions of the vkblas C API.
 *
 * These entry points have no counterpart in the reference's vkblas.h (its
 * engine was synchronous, single-stream and single-device).  They expose what
 * a stream-ordered CUDA library needs: a stream per calling thread, device
 * resident alpha/beta, kernel-path control for tests and benchmarks, the
 * device status word of the bounded waits, and the multi-GPU shard planner.
 */
#pragma once
#include "vkblas.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum { VKBLAS_DT_F32 = 0, VKBLAS_DT_F16 = 1, VKBLAS_DT_BF16 = 2 } vkblas_dtype_t;

/* Kernel families.  AUTO lets the dispatcher choose. */
typedef enum {
    VKBLAS_PATH_AUTO = 0,
    VKBLAS_PATH_SIMT = 1,   /* exact SIMT GEMM: sequential fp32 fmaf per output      */
    VKBLAS_PATH_TC = 2,     /* tcgen05 GEMM: kind::f16 (fp16/bf16) or 3xTF32 (fp32)   */
    VKBLAS_PATH_GEMV = 3    /* split-K decode GEMV (M <= 16, op_b == T, 2-byte types) */
} vkblas_path_t;

/* Generic entry used by the hipBLAS shim.  alpha and beta point to fp32
 * scalars in host memory (scalars_on_device == 0) or device memory (1); in
 * the device case the kernels read them, nothing is copied to the host.
 * stream: a cudaStream_t (NULL = legacy default stream). */
vkblas_status_t vkblas_gemm_ex(vkblas_dtype_t dtype, vkblas_op_t op_a, vkblas_op_t op_b,
                               uint32_t M, uint32_t N, uint32_t K,
                               const float* alpha, const float* beta, int scalars_on_device,
                               const void* A, uint32_t lda, const void* B, uint32_t ldb,
                               void* C, uint32_t ldc, uint32_t batch,
                               int64_t stride_a, int64_t stride_b, int64_t stride_c,
                               void* stream);

/* Frees this library's scratch workspaces on the current device: the ones
 * bound to `stream` (a cudaStream_t; NULL = legacy default stream) when
 * all == 0, or every stream's when all != 0.  Workspaces are grow-only and
 * kept per (device, stream) -- the 3xTF32 operand planes of a 4096^3 SGEMM
 * take 256 MB -- so a caller that ran GEMMs on many streams, or on a stream it
 * has destroyed, calls this to give the memory back; the next call that needs
 * scratch allocates it again.  Synchronises the device first.  Must not run
 * while another thread issues calls on this device.  Returns 0, or -1 when
 * no CUDA device state is available.  No counterpart in the reference. */
int vkblas_b200_release_workspaces(void* stream, int all);

/* Split-K decode GEMV that allocates nothing.  No counterpart in the
 * reference.  For callers that cannot let a library call cudaMalloc (work
 * inside a framework's allocator or memory pool, or decode loops where a
 * device-synchronising cudaFree/cudaMalloc of a growing workspace is not
 * acceptable).  Computes, for 2-byte dtype (VKBLAS_DT_F16 or VKBLAS_DT_BF16),
 *     C[m*ldc + n] = alpha * sum_k X[m*ldx + k] * W[n*ldw + k] + beta * C[m*ldc + n]
 * i.e. vkblas_gemm_f16/bf16(VKBLAS_OP_N, VKBLAS_OP_T, M, N, K, ...) with
 * batch 1, on `stream` (a cudaStream_t; NULL = legacy default stream), with
 * the K range split into `splitk` (1..16) segments.  Scratch is a fixed 4 MiB
 * array inside the library (held by every GPU that loads it until exit):
 * splitk*M*N*4 must fit in 4 MiB - 64 KiB and N in 16384*16 rows, and
 * M <= 16, K, ldx, ldw multiples of 8, X and W 16-byte aligned; otherwise
 * VKBLAS_ERR_PARAM and nothing is enqueued.  All calls on a device share the
 * array: calls whose kernels overlap on the GPU race (order them on one
 * stream).  The first call on a device looks the array up
 * (cudaGetSymbolAddress); make it before any stream capture. */
vkblas_status_t vkblas_gemv_splitk_noalloc(vkblas_dtype_t dtype, uint32_t M, uint32_t N,
                                           uint32_t K, float alpha, const void* X, uint32_t ldx,
                                           const void* W, uint32_t ldw, float beta, void* C,
                                           uint32_t ldc, uint32_t splitk, void* stream);

/* Replicated-output GEMM for data-parallel sharding.  No counterpart in the
 * reference (its engine drove one device).  Computes the engine call
 * (dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch,
 * stride_a/b/c) on the tcgen05 path, on `stream` (a cudaStream_t; NULL =
 * legacy default stream), and writes every element of C it produces also to
 * each of the `npeers` (0..7) buffers in peer_C, at the same element offset
 * from peer_C[j] as from C.  peer_C[j] are addresses valid in this process
 * (another GPU's memory mapped by CUDA IPC, over NVLink); the beta term reads
 * only C.  The peer stores are fenced system-wide before the kernels end;
 * the caller orders them before a peer reads its buffer with a collective
 * on `stream` after this call (a one-element NCCL all-reduce does).
 * VKBLAS_ERR_PARAM: unknown dtype, more than 7 peers, a null peer, or what
 * the engine rejects.  VKBLAS_ERR_FALLBACK (nothing launched, C and the
 * peers untouched): the problem cannot run on the tensor-core path (operand
 * alignment; a 2-byte problem with M <= 64 and N >= 128, which runs
 * transposed; scratch that cannot be had); the caller computes C and gathers
 * it another way. */
vkblas_status_t vkblas_b200_gemm_replicated(vkblas_dtype_t dtype, vkblas_op_t op_a,
                                            vkblas_op_t op_b, uint32_t M, uint32_t N, uint32_t K,
                                            float alpha, const void* A, uint32_t lda,
                                            const void* B, uint32_t ldb, float beta, void* C,
                                            uint32_t ldc, uint32_t batch, int64_t stride_a,
                                            int64_t stride_b, int64_t stride_c,
                                            void* const* peer_C, uint32_t npeers, void* stream);

/* Stream used by the vkblas_gemm_* calls made from the calling thread
 * (thread-local; default NULL = legacy default stream). */
void vkblas_set_stream(void* stream);
void* vkblas_get_stream(void);

/* Thread-local kernel-path override (VKBLAS_PATH_AUTO by default).  A forced
 * path that cannot run the call (alignment, shape) makes the call return
 * VKBLAS_ERR_FALLBACK instead of silently taking another path. */
void vkblas_b200_set_path(int path);
int vkblas_b200_get_path(void);
/* Path taken by the last successful call on this thread (vkblas_path_t). */
int vkblas_b200_last_path(void);
/* K-split count of that call: the GEMV split-K factor, or for the tensor-core
 * path the number of K ranges the tiles of its last, partial wave were cut
 * into (their partial sums are added by a second kernel); 1 = no split. */
int vkblas_b200_last_split(void);
/* 1 when that call ran on 2-CTA clusters (tcgen05 cta_group::2, 256-row
 * tiles: each CTA loads half of the B tile), else 0. */
int vkblas_b200_last_pair(void);
/* N width of that call's tensor-core tile: 256 for fp16/bf16 and for 3xTF32
 * on CTA pairs with N >= 256, 128 for other 3xTF32 tiles, 64 for small-M
 * transposed tiles (over the swapped problem); 0 when the call did not run on
 * the tensor-core path. */
int vkblas_b200_last_tile_n(void);
/* Thread-local split-K factor for the GEMV path: 0 = automatic, else 1..16. */
void vkblas_b200_set_splitk(int splitk);

/* Measurement hook (thread-local; NULL, NULL turns it off): while set, each
 * GEMM call made from this thread records the cudaEvent_t `start` on its
 * stream right before its main kernel (after the 3xTF32 split pre-pass, when
 * there is one) and `end` right after it (after the split-K reduce, when
 * there is one).  Timing those events gives the kernel's own duration inside
 * a stream of calls.  Both events must belong to the call's device. */
void vkblas_b200_set_kernel_events(void* start, void* end);

/* Device status word written by kernels whose bounded waits ran out (0 = no
 * error).  Synchronises the current device first.  clear != 0 resets it. */
int vkblas_b200_device_status(int clear);

/* Test hook for the bounded waits (thread-local, off by default): while on,
 * tcgen05 GEMMs launched from this thread leave their first shared-memory
 * stage unfilled and wait at most 20 ms, so the MMA warp's wait runs out, the
 * kernel records status 2 (MMA wait timeout) in the device status word and
 * every role unwinds; the context stays usable.  For tests only. */
void vkblas_b200_set_test_stall(int on);

/* Test hook for scratch-memory failure (thread-local, off by default): with
 * count > 0 the next `count` scratch requests made from this thread fail as a
 * failed cudaMalloc would, with count < 0 every request fails until the hook
 * is set to 0.  A call that then lacks its scratch runs without it where it
 * can (a GEMV or tensor-core GEMM without its K split; an fp32 GEMM on the
 * exact SIMT kernel instead of 3xTF32 when the path is automatic) or returns
 * VKBLAS_ERR_FALLBACK (path forced to VKBLAS_PATH_TC; the hipBLAS shim then
 * forwards the call).  For tests only. */
void vkblas_b200_set_test_alloc_fail(int count);

/* Number of kernels this library launched from the calling process (all
 * threads); used by tests and benchmarks to prove the native path ran. */
uint64_t vkblas_b200_launch_count(void);

/* Library version string. */
const char* vkblas_b200_version(void);

/* Tile and split plan of a tensor-core GEMM (pure host logic; no device is
 * touched).  For the engine call (dtype, op_a, op_b, M, N, K, batch) on a
 * device with `num_sms` SMs it reports the tiles the tcgen05 kernel would run
 * and how the tiles of the last, partial wave are cut along K.  allow_wide:
 * whether 256-wide 3xTF32 pair tiles may be chosen (the launch path allows
 * them when its kernel's register split fits and VKBLAS_TF32_WIDE is not 0).
 * The plan assumes the K-split is on (VKBLAS_TC_SPLIT) and its scratch can be
 * had.  Returns VKBLAS_ERR_PARAM for a zero size, num_sms < 1, an unknown dtype,
 * a null `out`, or 2^31 tiles or more (a call the tensor-core path rejects).
 * No counterpart in the reference. */
typedef struct {
    uint32_t tile_m;             /* rows of a tile: 128, or 256 on CTA pairs */
    uint32_t tile_n;             /* columns of a tile */
    uint32_t transposed;         /* 1: small-M 2-byte GEMM run as C^T = op(B)^T op(A)^T;
                                    tile_m, tile_n and tiles then refer to C^T */
    uint32_t pair;               /* 1: 2-CTA clusters (cta_group::2) */
    uint32_t tiles;              /* tiles over all batch entries */
    uint32_t full_tiles;         /* tiles computed whole (the full waves) */
    uint32_t splits;             /* K ranges each remaining tile is cut into; 1 = none */
    uint32_t kblocks;            /* k-blocks per tile: K / 32 (fp32) or K / 64, rounded up */
    uint32_t kblocks_per_split;  /* k-blocks per K range of a split tile */
    uint64_t partial_bytes;      /* fp32 partial-tile scratch of the split tiles */
    uint32_t tail_tiles;         /* tiles of the last wave run as two 256 x 128 halves each in a
                                    second, programmatically dependent grid (2-byte pair tiles
                                    whose last wave fills at most half the SM pairs); they
                                    follow the full_tiles whole tiles */
} vkblas_b200_tc_plan_t;
vkblas_status_t vkblas_b200_tc_plan(vkblas_dtype_t dtype, vkblas_op_t op_a, vkblas_op_t op_b,
                                    uint32_t M, uint32_t N, uint32_t K, uint32_t batch,
                                    int num_sms, int allow_wide, vkblas_b200_tc_plan_t* out);

/* Throughput microbenchmarks of the current device (no counterpart in the
 * reference's API; its test/fma_peak.c measured its FMA ceiling the same way).
 * Enqueues one launch of kernel `which` on `stream` (a cudaStream_t) that
 * runs `iters` rounds of only the instruction under test on every SM, and
 * stores the FLOP that launch performs in *flops; the caller times it with
 * CUDA events.  `status` is a device int that a bounded wait sets non-zero
 * if the tensor core's final commit never arrived.  VKBLAS_ERR_PARAM for an
 * unknown `which`, iters == 0 or null pointers; VKBLAS_ERR_INIT without an
 * sm_100 device. */
typedef enum {
    VKBLAS_PEAK_FFMA = 0,       /* fp32 fmaf, 2048 threads per SM                    */
    VKBLAS_PEAK_TF32 = 1,       /* tcgen05.mma kind::tf32, cta_group::1, 128x256x8   */
    VKBLAS_PEAK_TF32_PAIR = 2,  /* tcgen05.mma kind::tf32, cta_group::2, 256x256x8   */
    VKBLAS_PEAK_F16 = 3,        /* tcgen05.mma kind::f16,  cta_group::1, 128x256x16  */
    VKBLAS_PEAK_F16_PAIR = 4    /* tcgen05.mma kind::f16,  cta_group::2, 256x256x16  */
} vkblas_b200_peak_t;
vkblas_status_t vkblas_b200_peak_launch(int which, uint32_t iters, void* stream, int* status,
                                        double* flops);

/* Multi-GPU shard planner (pure host logic).  Splits `units` work units
 * (batch entries, or column blocks of `block` columns) into `world` contiguous
 * ranges as evenly as possible; returns this rank's [begin, begin+count).
 * Returns VKBLAS_ERR_PARAM for world < 1 or rank outside [0, world). */
vkblas_status_t vkblas_shard_range(uint64_t units, uint64_t block, int rank, int world,
                                   uint64_t* begin, uint64_t* count);

#ifdef __cplusplus
}
#endif
