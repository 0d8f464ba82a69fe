/* gemm_oracle.c -- CPU oracle for the vkblas GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker.
 *
 * It restates, in plain C, the arithmetic the reference (lakitu12/vkblas)
 * defines for its GEMM path:
 *
 *   - orc_sgemm_colmajor_f64acc: the reference's own CPU ground truth
 *     `ref_gemm` (test/test_gemm.c:32-58): hipBLAS column-major semantics,
 *     double accumulation, epilogue `alpha*(float)s + beta*C` in fp32.
 *   - orc_gemm_rowmajor_f32seq: the engine contract of src/vkblas.h:19-36
 *     (row-major C[M,N] = alpha*op(A)*op(B) + beta*C, beta==0 => C not read)
 *     computed the way the fp32 tile shaders do it: one fp32 accumulator per
 *     output, k visited in order, `acc += a*b` (fused here: fmaf), then
 *     `alpha*acc + beta*c` with separate roundings
 *     (src/shaders/gemm_f32_64x64_tmpl.comp:128-163).  This is the bit-exact
 *     target of the exact SIMT kernels.
 *   - orc_hgemm_rowmajor: the half-precision engine contract
 *     (vkblas.h:64-77, shader epilogue gemm_half_128x128_bankfree_tmpl.comp:
 *     203-228): 2-byte inputs widened to fp32, fp32 accumulate, fp32
 *     epilogue, round-to-nearest-even store.  acc_mode 0 accumulates in
 *     double (test/test_h.c:63-79), acc_mode 1 in sequential fp32 fmaf,
 *     acc_mode 2 in double with the reference test's own output encoder
 *     (test/test_h.c:23-41, ties rounded up) -- the exact pin of cpu_ref.
 *   - orc_hgemm_rowmajor_splitk: split-K semantics of the reference's
 *     matvec/split-K family (matvec_splitk_tmpl.comp:64-79,
 *     splitk_reduce_half.comp:22-35): per-segment fp32 partial sums, added in
 *     segment order, then alpha/beta and the store encoder: RNE (rounding 0,
 *     what this library's kernels do), or the reference reduce's own encoders
 *     (rounding 1: packHalf2x16 RNE for fp16, truncation to the upper 16 bits
 *     for bf16 -- splitk_reduce_half.comp:5,8, splitk_reduce_m_half.comp:6,9).
 *   - orc_dgemm_rowmajor_seq, orc_cgemm_rowmajor, orc_zgemm_rowmajor: the
 *     fp64 and complex fallbacks (src/vkblas.c:3653-4188): sequential fma in
 *     double; complex as four real GEMMs on planar copies plus the combine of
 *     cx_combine.comp / cx_combine_d64.comp.
 *   - orc_gemm_rowmajor_f32_splitk: the same segment model for fp32 (the
 *     decode matvec with K x N weights, matvec_f32_tmpl.comp TB=0).
 *   - f16/bf16 converters: exact RNE (what packHalf2x16 and the GPU's
 *     __float2half_rn do) plus a replica of test/test_h.c:16-41's own
 *     encoders, which the reference's tests use to build their inputs.
 *   - the reference tests' input generators (glibc srand/rand streams of
 *     test/test_gemm.c:70-73 and test/test_h.c:102-118).
 *
 * Must be compiled with -ffp-contract=off so that the epilogue's separate
 * roundings are kept.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#define EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------- helpers */

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Exact IEEE binary32 -> binary16, round to nearest, ties to even, with
 * subnormals, overflow to inf and NaN preserved (quietened). */
EXPORT uint16_t orc_f2h_rne(float f) {
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t e8 = (u >> 23) & 0xFFu;
    uint32_t man = u & 0x7FFFFFu;
    if (e8 == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u | (man >> 13) : 0u));
    int e = (int)e8 - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;            /* below half of the smallest subnormal */
        uint32_t m = man | 0x800000u;                   /* 24-bit significand */
        int shift = 14 - e;                             /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);                    /* a carry into the exponent is correct */
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;  /* carry may reach inf: correct */
    return (uint16_t)(sign | q);
}

EXPORT float orc_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (e == 0) {
        /* zero or subnormal: value = man * 2^-24, exact in fp32 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (e == 31) return bits_f32(sign | 0x7F800000u | (man << 13));
    return bits_f32(sign | ((e - 15 + 127) << 23) | (man << 13));
}

/* binary32 -> bfloat16, RNE; NaN kept NaN. */
EXPORT uint16_t orc_f2bf_rne(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

EXPORT float orc_bf2f(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* Replica of the reference test's own f16 encoder (test/test_h.c:23-41).
 * It rounds a tie upward instead of to even; the reference tests build their
 * fp16 inputs with it, so reproducing those inputs needs it. */
EXPORT uint16_t orc_f2h_test_h(float f) {
    uint32_t u = f32_bits(f);
    int sign = (u >> 16) & 0x8000;
    int exp8 = (u >> 23) & 0xFF, mant = u & 0x7FFFFF;
    int e = exp8 - 127 + 15;
    if (exp8 == 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7C00);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000;
        int shift = 14 - e;
        uint32_t half = (uint32_t)mant >> shift;
        if (((uint32_t)mant >> (shift - 1)) & 1u) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)e << 10) | ((uint32_t)mant >> 13);
    if (mant & 0x1000) half++;
    return (uint16_t)(sign | half);
}

static inline float widen(int dtype, uint16_t v) { return dtype ? orc_bf2f(v) : orc_h2f(v); }
static inline uint16_t narrow(int dtype, float v) { return dtype ? orc_f2bf_rne(v) : orc_f2h_rne(v); }
/* The reference test's own encoders (test/test_h.c:16-41): its bf16 encoder is
 * the RNE formula, its fp16 encoder rounds ties up. */
static inline uint16_t narrow_test_h(int dtype, float v) { return dtype ? orc_f2bf_rne(v) : orc_f2h_test_h(v); }

/* --------------------------------------------------- column-major, double */

/* ref_gemm semantics (test/test_gemm.c:32-58) over all rows. */
EXPORT void orc_sgemm_colmajor_f64acc(int transa, int transb, int m, int n, int k, float alpha,
                                      const float* A, int lda, const float* B, int ldb,
                                      float beta, float* C, int ldc) {
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            double s = 0.0;
            for (int t = 0; t < k; t++) {
                float av = transa ? A[t + (size_t)i * lda] : A[i + (size_t)t * lda];
                float bv = transb ? B[j + (size_t)t * ldb] : B[t + (size_t)j * ldb];
                s += (double)av * bv;
            }
            float* c = &C[i + (size_t)j * ldc];
            *c = alpha * (float)s + beta * *c;
        }
}

/* ------------------------------------------------------ row-major engine */

static inline size_t a_idx(int op_a, size_t m, size_t k, size_t lda) { return op_a ? k * lda + m : m * lda + k; }
static inline size_t b_idx(int op_b, size_t k, size_t n, size_t ldb) { return op_b ? n * ldb + k : k * ldb + n; }

EXPORT void orc_gemm_rowmajor_f32seq(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K,
                                     float alpha, const float* A, uint32_t lda,
                                     const float* B, uint32_t ldb, float beta,
                                     float* C, uint32_t ldc, uint32_t batch,
                                     int64_t sa, int64_t sb, int64_t sc) {
    for (uint32_t b = 0; b < batch; b++) {
        const float* Ab = A + sa * (int64_t)b;
        const float* Bb = B + sb * (int64_t)b;
        float* Cb = C + sc * (int64_t)b;
        for (uint32_t m = 0; m < M; m++)
            for (uint32_t n = 0; n < N; n++) {
                float acc = 0.0f;
                for (uint32_t k = 0; k < K; k++)
                    acc = fmaf(Ab[a_idx(op_a, m, k, lda)], Bb[b_idx(op_b, k, n, ldb)], acc);
                float* c = &Cb[(size_t)m * ldc + n];
                float old = beta != 0.0f ? *c : 0.0f;
                float t1 = alpha * acc;
                float t2 = beta * old;
                *c = t1 + t2;
            }
    }
}

/* The fp32 split-K matvec model (matvec_f32_tmpl.comp TB=0 per-output
 * sequential sums, split into segments and reduced in segment order as
 * splitk_reduce_f32.comp:61-69 does): K cut into segments of `span`; each
 * segment a sequential fmaf sum from +0; the segment sums added in order from
 * +0; then the fp32 epilogue with separate roundings.  span >= K is the
 * unsplit sequential contract. */
EXPORT void orc_gemm_rowmajor_f32_splitk(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K,
                                         uint32_t span, float alpha, const float* A,
                                         uint32_t lda, const float* B, uint32_t ldb,
                                         float beta, float* C, uint32_t ldc) {
    if (span == 0) span = K;
    for (uint32_t m = 0; m < M; m++)
        for (uint32_t n = 0; n < N; n++) {
            float total = 0.0f;
            for (uint32_t k0 = 0; k0 < K; k0 += span) {
                uint32_t k1 = k0 + span < K ? k0 + span : K;
                float part = 0.0f;
                for (uint32_t k = k0; k < k1; k++)
                    part = fmaf(A[a_idx(op_a, m, k, lda)], B[b_idx(op_b, k, n, ldb)], part);
                total += part;
            }
            float* c = &C[(size_t)m * ldc + n];
            float old = beta != 0.0f ? *c : 0.0f;
            float t1 = alpha * total;
            float t2 = beta * old;
            *c = t1 + t2;
        }
}

/* fp64 engine contract (gemm_f64_32x32_tmpl.comp:85-117): one double
 * accumulator per output, k in order with fma, then alpha*acc + beta*c with
 * separate roundings (c not read when beta == 0). */
EXPORT void orc_dgemm_rowmajor_seq(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K,
                                   double alpha, const double* A, uint32_t lda,
                                   const double* B, uint32_t ldb, double beta, double* C,
                                   uint32_t ldc, uint32_t batch, int64_t sa, int64_t sb,
                                   int64_t sc) {
    for (uint32_t b = 0; b < batch; b++) {
        const double* Ab = A + sa * (int64_t)b;
        const double* Bb = B + sb * (int64_t)b;
        double* Cb = C + sc * (int64_t)b;
        for (uint32_t m = 0; m < M; m++)
            for (uint32_t n = 0; n < N; n++) {
                double acc = 0.0;
                for (uint32_t k = 0; k < K; k++)
                    acc = fma(Ab[a_idx(op_a, m, k, lda)], Bb[b_idx(op_b, k, n, ldb)], acc);
                double* c = &Cb[(size_t)m * ldc + n];
                double old = beta != 0.0 ? *c : 0.0;
                double t1 = alpha * acc;
                double t2 = beta * old;
                *c = t1 + t2;
            }
    }
}

/* Complex GEMM the reference's way (src/vkblas.c:3748-3930, 4092-4188):
 * interleaved A, B, C split into real / imaginary planes at the same element
 * offsets, four real GEMMs
 *   T1 = Ar*Br;  T1 = -1*(Ai*Bi) + 1*T1;  T2 = Ar*Bi;  T2 = 1*(Ai*Br) + 1*T2
 * in the sequential engine contract (fp32 for complex64, fp64 for
 * complex128), then the combine of cx_combine.comp:32-45, left to right:
 *   C.r = ar*T1 - ai*T2 + br*C.r - bi*C.i,  C.i = ar*T2 + ai*T1 + br*C.i + bi*C.r
 * (the beta terms only when beta != 0). */
static size_t span_of(uint32_t rows, uint32_t cols, uint32_t ld, uint32_t batch, int64_t stride) {
    return (batch > 1 ? (size_t)stride * (batch - 1) : 0) + (size_t)(rows - 1) * ld + cols;
}

#define CX_GEMM_BODY(T, GEMM)                                                                  \
    uint32_t ra = op_a ? K : M, ca = op_a ? M : K, rb = op_b ? N : K, cb = op_b ? K : N;       \
    size_t ea = span_of(ra, ca, lda, batch, sa), eb = span_of(rb, cb, ldb, batch, sb);         \
    size_t ec = span_of(M, N, ldc, batch, sc);                                                 \
    T* Ar = (T*)calloc(ea, sizeof(T)); T* Ai = (T*)calloc(ea, sizeof(T));                      \
    T* Br = (T*)calloc(eb, sizeof(T)); T* Bi = (T*)calloc(eb, sizeof(T));                      \
    T* T1 = (T*)calloc(ec, sizeof(T)); T* T2 = (T*)calloc(ec, sizeof(T));                      \
    for (size_t i = 0; i < ea; i++) { Ar[i] = A[2 * i]; Ai[i] = A[2 * i + 1]; }                \
    for (size_t i = 0; i < eb; i++) { Br[i] = B[2 * i]; Bi[i] = B[2 * i + 1]; }                \
    GEMM(op_a, op_b, M, N, K, 1, Ar, lda, Br, ldb, 0, T1, ldc, batch, sa, sb, sc);             \
    GEMM(op_a, op_b, M, N, K, -1, Ai, lda, Bi, ldb, 1, T1, ldc, batch, sa, sb, sc);            \
    GEMM(op_a, op_b, M, N, K, 1, Ar, lda, Bi, ldb, 0, T2, ldc, batch, sa, sb, sc);             \
    GEMM(op_a, op_b, M, N, K, 1, Ai, lda, Br, ldb, 1, T2, ldc, batch, sa, sb, sc);             \
    for (uint32_t b = 0; b < batch; b++)                                                       \
        for (uint32_t m = 0; m < M; m++)                                                       \
            for (uint32_t n = 0; n < N; n++) {                                                 \
                size_t o = (size_t)(sc * (int64_t)b) + (size_t)m * ldc + n;                    \
                T fr = T1[o], fi = T2[o], outr, outi;                                          \
                if (br != 0 || bi != 0) {                                                      \
                    T r0 = C[2 * o], i0 = C[2 * o + 1];                                        \
                    outr = ar * fr - ai * fi + br * r0 - bi * i0;                              \
                    outi = ar * fi + ai * fr + br * i0 + bi * r0;                              \
                } else {                                                                       \
                    outr = ar * fr - ai * fi;                                                  \
                    outi = ar * fi + ai * fr;                                                  \
                }                                                                              \
                C[2 * o] = outr;                                                               \
                C[2 * o + 1] = outi;                                                           \
            }                                                                                  \
    free(Ar); free(Ai); free(Br); free(Bi); free(T1); free(T2);

EXPORT void orc_cgemm_rowmajor(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K, float ar,
                               float ai, const float* A, uint32_t lda, const float* B,
                               uint32_t ldb, float br, float bi, float* C, uint32_t ldc,
                               uint32_t batch, int64_t sa, int64_t sb, int64_t sc) {
    CX_GEMM_BODY(float, orc_gemm_rowmajor_f32seq)
}

EXPORT void orc_zgemm_rowmajor(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K, double ar,
                               double ai, const double* A, uint32_t lda, const double* B,
                               uint32_t ldb, double br, double bi, double* C, uint32_t ldc,
                               uint32_t batch, int64_t sa, int64_t sb, int64_t sc) {
    CX_GEMM_BODY(double, orc_dgemm_rowmajor_seq)
}

/* Double-precision product of the same contract, written to a separate
 * row-major M x N (tight) double buffer per batch: the error yardstick. */
EXPORT void orc_gemm_rowmajor_f64(int op_a, int op_b, uint32_t M, uint32_t N, uint32_t K,
                                  double alpha, const float* A, uint32_t lda,
                                  const float* B, uint32_t ldb, double beta,
                                  const float* Cin, uint32_t ldc, double* out,
                                  uint32_t batch, int64_t sa, int64_t sb, int64_t sc) {
    for (uint32_t b = 0; b < batch; b++) {
        const float* Ab = A + sa * (int64_t)b;
        const float* Bb = B + sb * (int64_t)b;
        const float* Cb = Cin ? Cin + sc * (int64_t)b : NULL;
        double* Ob = out + (size_t)b * M * N;
        for (uint32_t m = 0; m < M; m++)
            for (uint32_t n = 0; n < N; n++) {
                double s = 0.0;
                for (uint32_t k = 0; k < K; k++)
                    s += (double)Ab[a_idx(op_a, m, k, lda)] * (double)Bb[b_idx(op_b, k, n, ldb)];
                double old = (beta != 0.0 && Cb) ? (double)Cb[(size_t)m * ldc + n] : 0.0;
                Ob[(size_t)m * N + n] = alpha * s + beta * old;
            }
    }
}

EXPORT void orc_hgemm_rowmajor(int dtype, int acc_mode, int op_a, int op_b,
                               uint32_t M, uint32_t N, uint32_t K, float alpha,
                               const uint16_t* A, uint32_t lda, const uint16_t* B, uint32_t ldb,
                               float beta, uint16_t* C, uint32_t ldc, uint32_t batch,
                               int64_t sa, int64_t sb, int64_t sc) {
    for (uint32_t b = 0; b < batch; b++) {
        const uint16_t* Ab = A + sa * (int64_t)b;
        const uint16_t* Bb = B + sb * (int64_t)b;
        uint16_t* Cb = C + sc * (int64_t)b;
        for (uint32_t m = 0; m < M; m++)
            for (uint32_t n = 0; n < N; n++) {
                float accf;
                if (acc_mode == 0 || acc_mode == 2) {
                    double s = 0.0;
                    for (uint32_t k = 0; k < K; k++)
                        s += (double)widen(dtype, Ab[a_idx(op_a, m, k, lda)]) *
                             widen(dtype, Bb[b_idx(op_b, k, n, ldb)]);
                    accf = (float)s;
                } else {
                    accf = 0.0f;
                    for (uint32_t k = 0; k < K; k++)
                        accf = fmaf(widen(dtype, Ab[a_idx(op_a, m, k, lda)]),
                                    widen(dtype, Bb[b_idx(op_b, k, n, ldb)]), accf);
                }
                uint16_t* c = &Cb[(size_t)m * ldc + n];
                float old = beta != 0.0f ? widen(dtype, *c) : 0.0f;
                float t1 = alpha * accf;
                float t2 = beta * old;
                *c = acc_mode == 2 ? narrow_test_h(dtype, t1 + t2) : narrow(dtype, t1 + t2);
            }
    }
}

/* Split-K model: K cut into nseg segments of ceil(K/nseg); each segment is a
 * sequential fp32 sum; segment partials are added in segment order. */
static inline uint16_t narrow_reduce_ref(int dtype, float v) {
    if (!dtype) return orc_f2h_rne(v);
    uint32_t u;
    memcpy(&u, &v, 4);
    return (uint16_t)(u >> 16);          /* splitk_reduce_half.comp:8 */
}

EXPORT void orc_hgemm_rowmajor_splitk(int dtype, int op_a, int op_b, uint32_t M, uint32_t N,
                                      uint32_t K, uint32_t nseg, float alpha,
                                      const uint16_t* A, uint32_t lda, const uint16_t* B,
                                      uint32_t ldb, float beta, uint16_t* C, uint32_t ldc,
                                      int rounding) {
    uint32_t span = (K + nseg - 1) / nseg;
    for (uint32_t m = 0; m < M; m++)
        for (uint32_t n = 0; n < N; n++) {
            float total = 0.0f;
            for (uint32_t s = 0; s < nseg; s++) {
                uint32_t k0 = s * span, k1 = k0 + span < K ? k0 + span : K;
                float part = 0.0f;
                for (uint32_t k = k0; k < k1; k++)
                    part = fmaf(widen(dtype, A[a_idx(op_a, m, k, lda)]),
                                widen(dtype, B[b_idx(op_b, k, n, ldb)]), part);
                total += part;
            }
            uint16_t* c = &C[(size_t)m * ldc + n];
            float old = beta != 0.0f ? widen(dtype, *c) : 0.0f;
            float t1 = alpha * total;
            float t2 = beta * old;
            *c = rounding ? narrow_reduce_ref(dtype, t1 + t2) : narrow(dtype, t1 + t2);
        }
}

/* ------------------------------------------------------ input generators */

/* test/test_gemm.c:70-73: srand(seed) then A, B, C from (rand()%200-100)/10. */
EXPORT void orc_gen_test_gemm(unsigned seed, float* A, size_t na, float* B, size_t nb,
                              float* C, size_t nc) {
    srand(seed);
    for (size_t i = 0; i < na; i++) A[i] = (float)(rand() % 200 - 100) / 10.0f;
    for (size_t i = 0; i < nb; i++) B[i] = (float)(rand() % 200 - 100) / 10.0f;
    for (size_t i = 0; i < nc; i++) C[i] = (float)(rand() % 200 - 100) / 10.0f;
}

/* test/test_h.c:102-118 (single-matrix cases) and 170-186 (batched cases):
 * srand(seed); fp16 draws uniform [-1,1) through the test's own encoder; the
 * bf16 cases first draw (and discard) a stream of encoded zeros, then bf16
 * values, exactly as the test does. */
EXPORT void orc_gen_test_h(unsigned seed, int dtype, uint16_t* A, size_t na, uint16_t* B,
                           size_t nb, uint16_t* C, size_t nc, int batched) {
    srand(seed);
#define UNI() ((float)rand() / RAND_MAX * 2.0f - 1.0f)
    if (!batched) {
        for (size_t i = 0; i < na; i++) A[i] = orc_f2h_test_h(dtype == 0 ? UNI() : 0.0f);
        for (size_t i = 0; i < nb; i++) B[i] = orc_f2h_test_h(dtype == 0 ? UNI() : 0.0f);
        for (size_t i = 0; i < nc; i++) C[i] = orc_f2h_test_h(dtype == 0 ? UNI() : 0.0f);
    } else {
        for (size_t i = 0; i < na; i++) A[i] = orc_f2h_test_h(UNI());
        for (size_t i = 0; i < nb; i++) B[i] = orc_f2h_test_h(UNI());
        for (size_t i = 0; i < nc; i++) C[i] = orc_f2h_test_h(UNI());
    }
    if (dtype) {
        for (size_t i = 0; i < na; i++) A[i] = orc_f2bf_rne(UNI());
        for (size_t i = 0; i < nb; i++) B[i] = orc_f2bf_rne(UNI());
        for (size_t i = 0; i < nc; i++) C[i] = orc_f2bf_rne(UNI());
    }
#undef UNI
}

/* Row-sampled, multi-threaded timing harness for the column-major oracle:
 * rows [r0, r0+nr) of C split into contiguous blocks, one pthread each.  Used
 * only by bench.py's CPU-baseline leg when the reference build is absent. */
#include <pthread.h>
struct orc_rows_job {
    int transa, transb, n, k, lda, ldb, ldc, i0, cnt;
    float alpha, beta;
    const float *A, *B;
    float* C;
};
static void* orc_rows_worker(void* p) {
    struct orc_rows_job* j = (struct orc_rows_job*)p;
    const float* Ab = j->transa ? j->A + (size_t)j->i0 * j->lda : j->A + j->i0;
    orc_sgemm_colmajor_f64acc(j->transa, j->transb, j->cnt, j->n, j->k, j->alpha, Ab, j->lda,
                              j->B, j->ldb, j->beta, j->C + j->i0, j->ldc);
    return NULL;
}
EXPORT void orc_sgemm_colmajor_rows_mt(int transa, int transb, int m, int n, int k, float alpha,
                                       const float* A, int lda, const float* B, int ldb,
                                       float beta, float* C, int ldc, int r0, int nr,
                                       int threads) {
    (void)m;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    struct orc_rows_job jobs[256];
    pthread_t tid[256];
    int per = (nr + threads - 1) / threads, used = 0;
    for (int t = 0; t < threads; t++) {
        int cnt = nr - t * per;
        if (cnt > per) cnt = per;
        if (cnt <= 0) break;
        jobs[t] = (struct orc_rows_job){transa, transb, n, k, lda, ldb, ldc, r0 + t * per, cnt,
                                        alpha, beta, A, B, C};
        if (pthread_create(&tid[t], NULL, orc_rows_worker, &jobs[t]) != 0) {
            orc_rows_worker(&jobs[t]);
            tid[t] = 0;
        }
        used = t + 1;
    }
    for (int t = 0; t < used; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}
