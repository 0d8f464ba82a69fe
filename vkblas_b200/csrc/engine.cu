// engine.cu -- dispatcher and C API of the B200 BLAS core.
//
// Replaces the reference engine (lakitu12/vkblas src/vkblas.c): its Vulkan
// instance, pipelines, dma-buf import cache (src/ic_cache.h) and global
// submit-and-wait lock are gone.  Device pointers are used directly, work is
// enqueued on a CUDA stream, and the only shared state is a per-device record
// (SM count, status word) plus a grow-only workspace per (device, stream).
//
// Path selection (the reference's heuristics, src/vkblas.c:3104-3341 and
// 3517-3651, re-derived for B200):
//   1. 2-byte types, M <= 16, op_b == T, op_a == N, batch == 1 (decode
//      shapes, the reference's matvec family)  -> split-K GEMV (gemv.cu);
//   2. operands that satisfy TMA's alignment rules (16-byte aligned bases,
//      leading dimensions and batch strides)       -> tcgen05 GEMM
//      (umma_gemm.cu): kind::f16 for fp16/bf16, 3xTF32 for fp32;
//   3. anything else                              -> exact SIMT GEMM
//      (simt_gemm.cu), which accepts every op, ld and stride.
// Environment overrides, read once: VKBLAS_SGEMM=ffma|3xtf32|auto,
// VKBLAS_HGEMM=simt|tc|auto, VKBLAS_GEMV=0|1, VKBLAS_GEMV_SPLITK=n,
// VKBLAS_TC_SPLIT=0|1 (K-split of the tensor-core GEMM's last wave),
// VKBLAS_TC_PAIR=0|1 (256-row tiles on 2-CTA clusters; read in umma_gemm.cu),
// VKBLAS_TF32_WIDE=0|1 (256 x 256 3xTF32 pair tiles; read in umma_gemm.cu),
// VKBLAS_TRACE=1 (one line per call on stderr).
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "vkblas_b200.h"

namespace vkb {

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

struct Config {
    int sgemm = 0;      // 0 auto, 1 ffma (SIMT), 2 3xtf32 (TC)
    int hgemm = 0;      // 0 auto, 1 simt, 2 tc
    int gemv = 1;
    int gemv_splitk = 0;
    bool tc_split = true;
    bool trace = false;
};

const Config& config() {
    static Config c = [] {
        Config k;
        if (const char* e = getenv("VKBLAS_SGEMM")) {
            if (!strcmp(e, "ffma")) k.sgemm = 1;
            else if (!strcmp(e, "3xtf32")) k.sgemm = 2;
        }
        if (const char* e = getenv("VKBLAS_HGEMM")) {
            if (!strcmp(e, "simt")) k.hgemm = 1;
            else if (!strcmp(e, "tc")) k.hgemm = 2;
        }
        if (const char* e = getenv("VKBLAS_GEMV")) k.gemv = atoi(e) != 0;
        if (const char* e = getenv("VKBLAS_GEMV_SPLITK")) k.gemv_splitk = atoi(e);
        if (const char* e = getenv("VKBLAS_TC_SPLIT")) k.tc_split = atoi(e) != 0;
        k.trace = getenv("VKBLAS_TRACE") != nullptr;
        return k;
    }();
    return c;
}

struct Workspace {
    void* ptr = nullptr;
    size_t bytes = 0;
};

struct DeviceState {
    int dev = -1;
    int num_sms = 0;
    int cc_major = 0, cc_minor = 0;
    int* d_status = nullptr;
    std::mutex mu;
    // [0]: GEMV split-K (partials + zero-initialised tickets), [1]: 3xTF32 operand planes,
    // [2]: tcgen05 split-K partial tiles, [3]: complex GEMM planes.
    std::unordered_map<cudaStream_t, Workspace> ws[4];
};

std::mutex g_dev_mu;
DeviceState* g_devs[64] = {};

DeviceState* device_state(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_devs[dev]) return g_devs[dev];
    auto* d = new DeviceState();
    d->dev = dev;
    if (cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d->cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d->cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaMalloc(&d->d_status, sizeof(int)) != cudaSuccess ||
        cudaMemset(d->d_status, 0, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        delete d;
        return nullptr;
    }
    g_devs[dev] = d;
    return d;
}

// Test hook (vkblas_b200_set_test_alloc_fail): while non-zero, every scratch
// request made from this thread fails as a failed cudaMalloc would; a positive
// count runs down by one per request.
thread_local int tls_fail_alloc = 0;

// Grow-only scratch per (device, kind, stream).  Growth frees the old buffer
// (cudaFree waits for the device) and zero-fills the new one on the stream,
// which is what the GEMV split-K tickets need.  Not callable during stream
// capture: make one call of the largest shape before capturing.  Returns
// nullptr when the memory cannot be had; every caller then runs without the
// scratch (no split) or declines the call (the hipBLAS shim forwards it).
void* workspace(DeviceState* ds, int kind, cudaStream_t s, size_t bytes) {
    if (bytes == 0) return nullptr;
    if (tls_fail_alloc) {
        if (tls_fail_alloc > 0) tls_fail_alloc--;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(ds->mu);
    Workspace& w = ds->ws[kind][s];
    if (w.bytes >= bytes) return w.ptr;
    if (w.ptr) cudaFree(w.ptr);
    w.ptr = nullptr;
    w.bytes = 0;
    size_t want = bytes + bytes / 4;
    if (cudaMalloc(&w.ptr, want) != cudaSuccess) {
        cudaGetLastError();
        w.ptr = nullptr;
        return nullptr;
    }
    if (cudaMemsetAsync(w.ptr, 0, want, s) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(w.ptr);
        w.ptr = nullptr;
        return nullptr;
    }
    w.bytes = want;
    return w.ptr;
}

struct ThreadState {
    void* stream = nullptr;
    int path = VKBLAS_PATH_AUTO;
    int splitk = 0;
    int last = VKBLAS_PATH_AUTO;
    int last_split = 1;
    int last_pair = 0;
    int last_tile_n = 0;
    int test_stall = 0;
    // Measurement hook (vkblas_b200_set_kernel_events): recorded around the
    // main kernel of each call.
    void* ev_start = nullptr;
    void* ev_end = nullptr;
};
thread_local ThreadState tls;

const char* dtype_name(int d) { return d == DT_F32 ? "f32" : d == DT_F16 ? "f16" : "bf16"; }
const char* path_name(int p) {
    return p == VKBLAS_PATH_SIMT ? "simt" : p == VKBLAS_PATH_TC ? "tc" : p == VKBLAS_PATH_GEMV ? "gemv" : "auto";
}

vkblas_status_t check_problem(const GemmProblem& p) {
    if (p.M == 0 || p.N == 0 || p.K == 0 || p.batch == 0) return VKBLAS_ERR_PARAM;
    if (!p.A || !p.B || !p.C) return VKBLAS_ERR_PARAM;
    // Like the reference engine (src/vkblas.c:3114, 3528), leading dimensions
    // are not checked against the matrix extents: a smaller ld makes rows
    // overlap, which the reference's own tests use (test/test_h.c:105 with
    // op_a == T) and which the SIMT kernel computes exactly as addressed.
    if (p.sa < 0 || p.sb < 0 || p.sc < 0) return VKBLAS_ERR_PARAM;
    return VKBLAS_OK;
}

vkblas_status_t run(GemmProblem& p, cudaStream_t s) {
    vkblas_status_t st = check_problem(p);
    if (st != VKBLAS_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    DeviceState* ds = device_state(dev);
    if (!ds || ds->cc_major != 10) return VKBLAS_ERR_INIT;
    const Config& cfg = config();
    const int forced = tls.path;

    int path = 0;
    if ((forced == VKBLAS_PATH_AUTO && cfg.gemv) || forced == VKBLAS_PATH_GEMV) {
        // Every 2-byte decode shape the GEMV takes (M <= 16) runs on it.  The
        // small-M tcgen05 GEMM was as fast at 9-16 tokens on some boxes
        // (4096 -> 14336, M = 16: 23.2 against 23.5 us) and far slower on
        // others (33.5 against 23.6 us); the GEMV held 23.5 us on both.
        if (gemv_supported(p)) path = VKBLAS_PATH_GEMV;
        // fp32 decode GEMV, unless the exact FFMA kernel was asked for
        else if (gemv_f32_supported(p) && (forced == VKBLAS_PATH_GEMV || cfg.sgemm != 1))
            path = VKBLAS_PATH_GEMV;
    }
    if (!path && (forced == VKBLAS_PATH_AUTO || forced == VKBLAS_PATH_TC)) {
        const int mode = p.dtype == DT_F32 ? cfg.sgemm : cfg.hgemm;   // 0 auto, 1 simt, 2 tc
        bool allow = forced == VKBLAS_PATH_TC || mode == 2 || (mode == 0 && umma_profitable(p));
        if (allow && umma_supported(p)) path = VKBLAS_PATH_TC;
    }
    if (!path && (forced == VKBLAS_PATH_AUTO || forced == VKBLAS_PATH_SIMT)) path = VKBLAS_PATH_SIMT;
    if (!path) return VKBLAS_ERR_FALLBACK;

    cudaError_t e = cudaSuccess;
    int splitk = 0, split_used = 1, pair_used = 0, tile_n = 0;
    const cudaEvent_t ev0 = reinterpret_cast<cudaEvent_t>(tls.ev_start);
    const cudaEvent_t ev1 = reinterpret_cast<cudaEvent_t>(tls.ev_end);
    auto rec = [&](cudaEvent_t ev) {
        if (ev) cudaEventRecord(ev, s);
    };
    if (path == VKBLAS_PATH_GEMV && p.dtype == DT_F32) {
        splitk = tls.splitk > 0 ? tls.splitk : cfg.gemv_splitk > 0 ? cfg.gemv_splitk
                                                                   : gemv_f32_auto_splitk(p, ds->num_sms);
        if (splitk > 64) splitk = 64;
        void* ws = nullptr;
        const size_t need = gemv_f32_workspace_bytes(p, splitk);
        if (need) {
            ws = workspace(ds, 0, s, need);
            if (!ws) splitk = 1;
        }
        rec(ev0);
        e = launch_gemv_f32(p, splitk, ws, s);
        rec(ev1);
        split_used = splitk;
    } else if (path == VKBLAS_PATH_GEMV) {
        splitk = tls.splitk > 0 ? tls.splitk : cfg.gemv_splitk > 0 ? cfg.gemv_splitk
                                                                   : gemv_auto_splitk(p, ds->num_sms);
        if (splitk > 16) splitk = 16;
        void* ws = nullptr;
        size_t need = gemv_workspace_bytes(p, splitk);
        if (need) {
            ws = workspace(ds, 0, s, need);
            if (!ws) splitk = 1;
        }
        rec(ev0);
        e = launch_gemv(p, splitk, ws, ds->d_status, s);
        split_used = splitk;
        if (e == cudaErrorNotSupported && forced == VKBLAS_PATH_AUTO) {
            cudaGetLastError();
            path = VKBLAS_PATH_SIMT;       // weights TMA cannot describe: exact SIMT path
            split_used = 1;
            e = launch_simt_gemm(p, s);
        } else if (e == cudaErrorNotSupported) {
            cudaGetLastError();
            return VKBLAS_ERR_FALLBACK;
        }
        rec(ev1);
    } else if (path == VKBLAS_PATH_TC) {
        const size_t need = umma_workspace_bytes(p);
        void* ws = need ? workspace(ds, 1, s, need) : nullptr;
        const size_t need_split = cfg.tc_split ? umma_split_workspace_bytes(p, ds->num_sms) : 0;
        void* wsplit = need_split ? workspace(ds, 2, s, need_split) : nullptr;   // null: no split
        e = (need && !ws) ? cudaErrorNotSupported
                          : launch_umma_gemm(p, ds->num_sms, ds->d_status, ws, wsplit,
                                             tls.test_stall != 0, s, ev0, ev1);
        split_used = wsplit ? umma_split_count(p, ds->num_sms) : 1;
        pair_used = umma_uses_pair(p, ds->num_sms, wsplit != nullptr) ? 1 : 0;
        tile_n = umma_tile_n(p);
        if (e == cudaErrorNotSupported && forced == VKBLAS_PATH_AUTO) {
            cudaGetLastError();
            path = VKBLAS_PATH_SIMT;       // operands TMA cannot describe: exact SIMT path
            split_used = 1;
            pair_used = 0;
            tile_n = 0;
            rec(ev0);
            e = launch_simt_gemm(p, s);
            rec(ev1);
        } else if (e == cudaErrorNotSupported) {
            cudaGetLastError();
            return VKBLAS_ERR_FALLBACK;
        }
    } else {
        rec(ev0);
        e = launch_simt_gemm(p, s);
        rec(ev1);
    }
    if (cfg.trace)
        fprintf(stderr, "[vkblas] gemm %s %c%c M=%u N=%u K=%u lda=%u ldb=%u ldc=%u batch=%u path=%s%s%d -> %s\n",
                dtype_name(p.dtype), p.op_a ? 'T' : 'N', p.op_b ? 'T' : 'N', p.M, p.N, p.K, p.lda,
                p.ldb, p.ldc, p.batch, path_name(path), path == VKBLAS_PATH_GEMV ? " splitk=" : " ",
                path == VKBLAS_PATH_GEMV ? splitk : 0, cudaGetErrorString(e));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration ? VKBLAS_ERR_PARAM
                                                                                 : VKBLAS_ERR_INIT;
    }
    tls.last = path;
    tls.last_split = split_used;
    tls.last_pair = pair_used;
    tls.last_tile_n = tile_n;
    return VKBLAS_OK;
}

GemmProblem make_problem(int dtype, vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N,
                         uint32_t K, float alpha, const void* A, uint32_t lda, const void* B,
                         uint32_t ldb, float beta, void* C, uint32_t ldc, uint32_t batch,
                         int64_t sa, int64_t sb, int64_t sc) {
    GemmProblem p;
    p.dtype = dtype;
    p.op_a = op_a == VKBLAS_OP_T;
    p.op_b = op_b == VKBLAS_OP_T;
    p.M = M; p.N = N; p.K = K;
    p.alpha = alpha; p.beta = beta;
    p.d_alpha = nullptr; p.d_beta = nullptr;
    p.A = A; p.lda = lda; p.B = B; p.ldb = ldb; p.C = C; p.ldc = ldc;
    p.batch = batch;
    // A batch of one never steps: normalise its strides.
    p.sa = batch > 1 ? sa : 0; p.sb = batch > 1 ? sb : 0; p.sc = batch > 1 ? sc : 0;
    return p;
}

}  // namespace
}  // namespace vkb

using namespace vkb;

#define VKB_EXPORT extern "C" __attribute__((visibility("default")))

VKB_EXPORT void vkblas_cache_invalidate_base(const void* ptr) { (void)ptr; }

VKB_EXPORT vkblas_status_t vkblas_gemm_f32(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M,
                                           uint32_t N, uint32_t K, float alpha, const void* A,
                                           uint32_t lda, const void* B, uint32_t ldb, float beta,
                                           void* C, uint32_t ldc, uint32_t batch,
                                           int64_t stride_a, int64_t stride_b, int64_t stride_c) {
    GemmProblem p = make_problem(DT_F32, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                                 batch, stride_a, stride_b, stride_c);
    return run(p, reinterpret_cast<cudaStream_t>(tls.stream));
}

VKB_EXPORT vkblas_status_t vkblas_gemm_f16(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M,
                                           uint32_t N, uint32_t K, float alpha, const void* A,
                                           uint32_t lda, const void* B, uint32_t ldb, float beta,
                                           void* C, uint32_t ldc, uint32_t batch,
                                           int64_t stride_a, int64_t stride_b, int64_t stride_c) {
    GemmProblem p = make_problem(DT_F16, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                                 batch, stride_a, stride_b, stride_c);
    return run(p, reinterpret_cast<cudaStream_t>(tls.stream));
}

VKB_EXPORT vkblas_status_t vkblas_gemm_bf16(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M,
                                            uint32_t N, uint32_t K, float alpha, const void* A,
                                            uint32_t lda, const void* B, uint32_t ldb, float beta,
                                            void* C, uint32_t ldc, uint32_t batch,
                                            int64_t stride_a, int64_t stride_b, int64_t stride_c) {
    GemmProblem p = make_problem(DT_BF16, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                                 batch, stride_a, stride_b, stride_c);
    return run(p, reinterpret_cast<cudaStream_t>(tls.stream));
}

VKB_EXPORT vkblas_status_t vkblas_gemm_bf16_hipblas(vkblas_op_t op_a, vkblas_op_t op_b,
                                                    uint32_t M, uint32_t N, uint32_t K,
                                                    float alpha, const void* A, uint32_t lda,
                                                    const void* B, uint32_t ldb, float beta,
                                                    void* C, uint32_t ldc, uint32_t batch,
                                                    int64_t stride_a, int64_t stride_b,
                                                    int64_t stride_c) {
    return vkblas_gemm_bf16(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch,
                            stride_a, stride_b, stride_c);
}

// ---------------------------------------------- fp64 and complex GEMMs
// Reference src/vkblas.c:3748-4188: fp64 runs one exact fp64 GEMM; complex64
// and complex128 run four real GEMMs on planar copies and a combine (see
// dgemm.cu for the arithmetic).  0 = done; non-zero = not run (the caller
// forwards to a real library), as in the reference.

namespace {

// Elements an operand spans: (batch - 1) * stride + (rows - 1) * ld + cols.
size_t extent(uint32_t rows, uint32_t cols, uint32_t ld, uint32_t batch, int64_t stride) {
    return (size_t)(batch > 1 ? (size_t)stride * (batch - 1) : 0) + (size_t)(rows - 1) * ld + cols;
}

DeviceState* current_device(cudaStream_t& s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    DeviceState* ds = device_state(dev);
    if (!ds || ds->cc_major != 10) return nullptr;
    s = reinterpret_cast<cudaStream_t>(tls.stream);
    return ds;
}

bool valid_batched(uint32_t M, uint32_t N, uint32_t K, uint32_t batch, const void* A,
                   const void* B, const void* C, int64_t sa, int64_t sb, int64_t sc) {
    return M && N && K && batch && A && B && C && sa >= 0 && sb >= 0 && sc >= 0;
}

// Complex GEMM through planar copies: four real GEMMs (fp32 engine calls or
// fp64 kernels) and the combine, all on stream s.
int complex_gemm(bool dbl, vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N, uint32_t K,
                 double ar, double ai, const void* A, uint32_t lda, const void* B, uint32_t ldb,
                 double br, double bi, void* C, uint32_t ldc, uint32_t batch, int64_t sa,
                 int64_t sb, int64_t sc) {
    if (!valid_batched(M, N, K, batch, A, B, C, sa, sb, sc)) return 1;
    cudaStream_t s;
    DeviceState* ds = current_device(s);
    if (!ds) return 1;
    const size_t es = dbl ? 8 : 4;
    const uint32_t ra = op_a ? K : M, ca = op_a ? M : K;
    const uint32_t rb = op_b ? N : K, cb = op_b ? K : N;
    const size_t ea = extent(ra, ca, lda, batch, sa), eb = extent(rb, cb, ldb, batch, sb);
    const size_t ec = extent(M, N, ldc, batch, sc);
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t need = 2 * (up(ea * es) + up(eb * es) + up(ec * es));
    char* w = static_cast<char*>(workspace(ds, 3, s, need));
    if (!w) return 1;
    void* Ar = w;
    void* Ai = w + up(ea * es);
    void* Br = w + 2 * up(ea * es);
    void* Bi = static_cast<char*>(Br) + up(eb * es);
    void* T1 = static_cast<char*>(Bi) + up(eb * es);
    void* T2 = static_cast<char*>(T1) + up(ec * es);
    if (launch_cx_split(dbl, A, ra, ca, lda, sa, batch, Ar, Ai, s) != cudaSuccess ||
        launch_cx_split(dbl, B, rb, cb, ldb, sb, batch, Br, Bi, s) != cudaSuccess)
        return 1;
    // T1 = Ar Br; T1 = -(Ai Bi) + T1; T2 = Ar Bi; T2 = Ai Br + T2  (src/vkblas.c:3816-3823)
    const void* As[4] = {Ar, Ai, Ar, Ai};
    const void* Bs[4] = {Br, Bi, Bi, Br};
    void* Cs[4] = {T1, T1, T2, T2};
    const double al[4] = {1.0, -1.0, 1.0, 1.0}, be[4] = {0.0, 1.0, 0.0, 1.0};
    for (int i = 0; i < 4; i++) {
        if (dbl) {
            if (launch_dgemm(op_a, op_b, M, N, K, al[i], static_cast<const double*>(As[i]), lda,
                             static_cast<const double*>(Bs[i]), ldb, be[i],
                             static_cast<double*>(Cs[i]), ldc, batch, sa, sb, sc, s) != cudaSuccess)
                return 1;
        } else {
            GemmProblem p = make_problem(DT_F32, op_a, op_b, M, N, K, (float)al[i], As[i], lda, Bs[i],
                                         ldb, (float)be[i], Cs[i], ldc, batch, sa, sb, sc);
            if (run(p, s) != VKBLAS_OK) return 1;
        }
    }
    return launch_cx_combine(dbl, T1, T2, C, M, N, ldc, sc, batch, ar, ai, br, bi, s) == cudaSuccess
               ? 0
               : 1;
}

}  // namespace

VKB_EXPORT int vkblas_gemm_c64(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N,
                               uint32_t K, float alpha_r, float alpha_i, const void* A,
                               uint32_t lda, const void* B, uint32_t ldb, float beta_r,
                               float beta_i, void* C, uint32_t ldc, uint32_t batch,
                               int64_t stride_a, int64_t stride_b, int64_t stride_c) {
    return complex_gemm(false, op_a, op_b, M, N, K, alpha_r, alpha_i, A, lda, B, ldb, beta_r,
                        beta_i, C, ldc, batch, stride_a, stride_b, stride_c);
}

VKB_EXPORT int vkblas_gemm_f64(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N,
                               uint32_t K, double alpha, const void* A, uint32_t lda,
                               const void* B, uint32_t ldb, double beta, void* C, uint32_t ldc,
                               uint32_t batch, int64_t stride_a, int64_t stride_b,
                               int64_t stride_c) {
    if (!valid_batched(M, N, K, batch, A, B, C, stride_a, stride_b, stride_c)) return 1;
    cudaStream_t s;
    if (!current_device(s)) return 1;
    return launch_dgemm(op_a, op_b, M, N, K, alpha, static_cast<const double*>(A), lda,
                        static_cast<const double*>(B), ldb, beta, static_cast<double*>(C), ldc,
                        batch, stride_a, stride_b, stride_c, s) == cudaSuccess
               ? 0
               : 1;
}

VKB_EXPORT int vkblas_gemm_z64(vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N,
                               uint32_t K, double alpha_r, double alpha_i, const void* A,
                               uint32_t lda, const void* B, uint32_t ldb, double beta_r,
                               double beta_i, void* C, uint32_t ldc, uint32_t batch,
                               int64_t stride_a, int64_t stride_b, int64_t stride_c) {
    return complex_gemm(true, op_a, op_b, M, N, K, alpha_r, alpha_i, A, lda, B, ldb, beta_r, beta_i,
                        C, ldc, batch, stride_a, stride_b, stride_c);
}

VKB_EXPORT vkblas_status_t vkblas_gemm_ex(vkblas_dtype_t dtype, vkblas_op_t op_a, vkblas_op_t op_b,
                                          uint32_t M, uint32_t N, uint32_t K, const float* alpha,
                                          const float* beta, int scalars_on_device, const void* A,
                                          uint32_t lda, const void* B, uint32_t ldb, void* C,
                                          uint32_t ldc, uint32_t batch, int64_t stride_a,
                                          int64_t stride_b, int64_t stride_c, void* stream) {
    if (!alpha || !beta) return VKBLAS_ERR_PARAM;
    if (dtype != VKBLAS_DT_F32 && dtype != VKBLAS_DT_F16 && dtype != VKBLAS_DT_BF16)
        return VKBLAS_ERR_PARAM;
    GemmProblem p = make_problem((int)dtype, op_a, op_b, M, N, K, 0.f, A, lda, B, ldb, 0.f, C, ldc,
                                 batch, stride_a, stride_b, stride_c);
    if (scalars_on_device) {
        p.d_alpha = alpha;
        p.d_beta = beta;
    } else {
        p.alpha = *alpha;
        p.beta = *beta;
    }
    return run(p, reinterpret_cast<cudaStream_t>(stream));
}

// Tensor-core GEMM whose epilogue also writes every C element it computes to
// up to 7 peer copies of C (replicated output for data-parallel sharding: each
// rank computes its shard and stores it into every rank's full buffer over
// NVLink).  No counterpart in the reference (single device).
VKB_EXPORT vkblas_status_t vkblas_b200_gemm_replicated(
    vkblas_dtype_t dtype, vkblas_op_t op_a, vkblas_op_t op_b, uint32_t M, uint32_t N, uint32_t K,
    float alpha, const void* A, uint32_t lda, const void* B, uint32_t ldb, float beta, void* C,
    uint32_t ldc, uint32_t batch, int64_t stride_a, int64_t stride_b, int64_t stride_c,
    void* const* peer_C, uint32_t npeers, void* stream) {
    if (dtype != VKBLAS_DT_F32 && dtype != VKBLAS_DT_F16 && dtype != VKBLAS_DT_BF16)
        return VKBLAS_ERR_PARAM;
    if (npeers > 7 || (npeers && !peer_C)) return VKBLAS_ERR_PARAM;
    for (uint32_t j = 0; j < npeers; j++)
        if (!peer_C[j]) return VKBLAS_ERR_PARAM;
    GemmProblem p = make_problem((int)dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C,
                                 ldc, batch, stride_a, stride_b, stride_c);
    vkblas_status_t st = check_problem(p);
    if (st != VKBLAS_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return VKBLAS_ERR_INIT;
    }
    DeviceState* ds = device_state(dev);
    if (!ds || ds->cc_major != 10) return VKBLAS_ERR_INIT;
    if (!umma_supported(p)) return VKBLAS_ERR_FALLBACK;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const Config& cfg = config();
    const size_t need = umma_workspace_bytes(p);
    void* ws = need ? workspace(ds, 1, s, need) : nullptr;
    if (need && !ws) return VKBLAS_ERR_FALLBACK;
    const size_t need_split = cfg.tc_split ? umma_split_workspace_bytes(p, ds->num_sms) : 0;
    void* wsplit = need_split ? workspace(ds, 2, s, need_split) : nullptr;   // null: no split
    cudaError_t e = launch_umma_gemm(p, ds->num_sms, ds->d_status, ws, wsplit, tls.test_stall != 0,
                                     s, reinterpret_cast<cudaEvent_t>(tls.ev_start),
                                     reinterpret_cast<cudaEvent_t>(tls.ev_end), peer_C, npeers);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e == cudaErrorNotSupported ? VKBLAS_ERR_FALLBACK
               : e == cudaErrorInvalidValue ? VKBLAS_ERR_PARAM : VKBLAS_ERR_INIT;
    }
    tls.last = VKBLAS_PATH_TC;
    tls.last_split = wsplit ? umma_split_count(p, ds->num_sms) : 1;
    tls.last_pair = umma_uses_pair(p, ds->num_sms, wsplit != nullptr) ? 1 : 0;
    tls.last_tile_n = umma_tile_n(p);
    return VKBLAS_OK;
}

VKB_EXPORT void vkblas_set_stream(void* stream) { tls.stream = stream; }
VKB_EXPORT void* vkblas_get_stream(void) { return tls.stream; }
VKB_EXPORT void vkblas_b200_set_path(int path) {
    tls.path = (path >= VKBLAS_PATH_AUTO && path <= VKBLAS_PATH_GEMV) ? path : VKBLAS_PATH_AUTO;
}
VKB_EXPORT int vkblas_b200_get_path(void) { return tls.path; }
VKB_EXPORT int vkblas_b200_last_path(void) { return tls.last; }
VKB_EXPORT int vkblas_b200_last_split(void) { return tls.last_split; }
VKB_EXPORT int vkblas_b200_last_pair(void) { return tls.last_pair; }
VKB_EXPORT int vkblas_b200_last_tile_n(void) { return tls.last_tile_n; }
VKB_EXPORT void vkblas_b200_set_splitk(int splitk) {
    tls.splitk = splitk < 0 ? 0 : splitk > 16 ? 16 : splitk;
}

VKB_EXPORT void vkblas_b200_set_test_stall(int on) { tls.test_stall = on ? 1 : 0; }

VKB_EXPORT void vkblas_b200_set_test_alloc_fail(int count) { tls_fail_alloc = count; }

VKB_EXPORT void vkblas_b200_set_kernel_events(void* start, void* end) {
    tls.ev_start = start;
    tls.ev_end = end;
}

VKB_EXPORT int vkblas_b200_device_status(int clear) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    DeviceState* ds = device_state(dev);
    if (!ds) return -1;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    int v = 0;
    if (cudaMemcpy(&v, ds->d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    if (clear) cudaMemset(ds->d_status, 0, sizeof(int));
    return v;
}

VKB_EXPORT int vkblas_b200_release_workspaces(void* stream, int all) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    DeviceState* ds = device_state(dev);
    if (!ds) return -1;
    // Queued kernels may still use the buffers.
    if (cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    std::lock_guard<std::mutex> lk(ds->mu);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (auto& kind : ds->ws) {
        for (auto it = kind.begin(); it != kind.end();) {
            if (all || it->first == s) {
                if (it->second.ptr) cudaFree(it->second.ptr);
                it = kind.erase(it);
            } else {
                ++it;
            }
        }
    }
    return 0;
}

VKB_EXPORT uint64_t vkblas_b200_launch_count(void) { return g_launches.load(); }

VKB_EXPORT const char* vkblas_b200_version(void) { return "vkblas-b200 0.1 (sm_100a)"; }

VKB_EXPORT vkblas_status_t vkblas_b200_tc_plan(vkblas_dtype_t dtype, vkblas_op_t op_a,
                                               vkblas_op_t op_b, uint32_t M, uint32_t N,
                                               uint32_t K, uint32_t batch, int num_sms,
                                               int allow_wide, vkblas_b200_tc_plan_t* out) {
    if (!out || !M || !N || !K || !batch || num_sms < 1) return VKBLAS_ERR_PARAM;
    if (dtype != VKBLAS_DT_F32 && dtype != VKBLAS_DT_F16 && dtype != VKBLAS_DT_BF16)
        return VKBLAS_ERR_PARAM;
    // Only sizes, types and ops shape the plan; pointers and leading dimensions do not.
    GemmProblem p = make_problem((int)dtype, op_a, op_b, M, N, K, 1.f, nullptr, 0, nullptr, 0, 0.f,
                                 nullptr, 0, batch, 0, 0, 0);
    const UmmaPlan r = umma_plan(p, num_sms, allow_wide != 0);
    if (r.too_many_tiles) return VKBLAS_ERR_PARAM;     // the launch path rejects such a call too
    out->tile_m = r.tile_m;
    out->tile_n = r.tile_n;
    out->transposed = r.transposed;
    out->pair = r.pair;
    out->tiles = r.tiles;
    out->full_tiles = r.full_tiles;
    out->splits = r.splits;
    out->kblocks = r.kblocks;
    out->kblocks_per_split = r.kblocks_per_split;
    out->partial_bytes = r.partial_bytes;
    out->tail_tiles = r.tail_tiles;
    return VKBLAS_OK;
}

VKB_EXPORT vkblas_status_t vkblas_shard_range(uint64_t units, uint64_t block, int rank, int world,
                                              uint64_t* begin, uint64_t* count) {
    if (world < 1 || rank < 0 || rank >= world || !begin || !count) return VKBLAS_ERR_PARAM;
    if (block == 0) block = 1;
    const uint64_t nblk = (units + block - 1) / block;
    const uint64_t base = nblk / (uint64_t)world, rem = nblk % (uint64_t)world;
    const uint64_t r = (uint64_t)rank;
    const uint64_t b0 = r * base + (r < rem ? r : rem);
    const uint64_t nb = base + (r < rem ? 1 : 0);
    uint64_t lo = b0 * block, hi = (b0 + nb) * block;
    if (lo > units) lo = units;
    if (hi > units) hi = units;
    *begin = lo;
    *count = hi - lo;
    return VKBLAS_OK;
}
