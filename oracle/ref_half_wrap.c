/* ref_half_wrap.c -- compiles the reference's own half-precision CPU checker
 * (test/test_h.c of lakitu12/vkblas, included by path at build time, never
 * copied) into oracle/_ref/libvkref.so.
 *
 * TEST INFRASTRUCTURE ONLY.  The reference's main() is renamed and never run.
 */
#include <stdint.h>
#define main vkref_unused_test_h_main
#include REF_TEST_H_C
#undef main

#define EXPORT __attribute__((visibility("default")))

/* test/test_h.c:63-79, called unmodified. dtype 0 = fp16, 1 = bf16. */
EXPORT void vkref_cpu_ref_half(int dtype, int op_a, int op_b, int M, int N, int K,
                               const uint16_t* A, int lda, const uint16_t* B, int ldb,
                               float alpha, float beta, uint16_t* C, int ldc) {
    cpu_ref(dtype, op_a, op_b, M, N, K, A, lda, B, ldb, alpha, beta, C, ldc);
}
/* test/test_h.c:16-60 converters. */
EXPORT uint16_t vkref_f2h(float f) { return f2h(f); }
EXPORT float vkref_h2f(uint16_t h) { return h2f(h); }
EXPORT uint16_t vkref_f2bf(float f) { return f2bf(f); }
EXPORT float vkref_bf2f(uint16_t b) { return bf2f(b); }

/* All-core timing harness for cpu_ref: columns [c0, c0+nc) of row-major C are
 * split into contiguous blocks and each pthread calls the unmodified cpu_ref
 * on its block (B offset n0*ldb for op_b T, n0 for op_b N; C offset n0).
 * Splitting columns, not rows, keeps every thread busy for a decode GEMM with
 * a single row. */
#include <pthread.h>
struct vkref_hjob {
    int dtype, op_a, op_b, M, K, lda, ldb, ldc, n0, cnt;
    float alpha, beta;
    const uint16_t *A, *B;
    uint16_t* C;
};
static void* vkref_hworker(void* p) {
    struct vkref_hjob* j = (struct vkref_hjob*)p;
    const uint16_t* Bb = j->op_b ? j->B + (size_t)j->n0 * j->ldb : j->B + j->n0;
    cpu_ref(j->dtype, j->op_a, j->op_b, j->M, j->cnt, j->K, j->A, j->lda, Bb, j->ldb, j->alpha,
            j->beta, j->C + j->n0, j->ldc);
    return NULL;
}
EXPORT void vkref_cpu_ref_half_cols_mt(int dtype, int op_a, int op_b, int M, int N, int K,
                                       const uint16_t* A, int lda, const uint16_t* B, int ldb,
                                       float alpha, float beta, uint16_t* C, int ldc, int c0,
                                       int nc, int threads) {
    (void)N;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    struct vkref_hjob jobs[256];
    pthread_t tid[256];
    int per = (nc + threads - 1) / threads, used = 0;
    for (int t = 0; t < threads; t++) {
        int cnt = nc - t * per;
        if (cnt > per) cnt = per;
        if (cnt <= 0) break;
        jobs[t] = (struct vkref_hjob){dtype, op_a, op_b, M, K, lda, ldb, ldc, c0 + t * per, cnt,
                                      alpha, beta, A, B, C};
        if (pthread_create(&tid[t], NULL, vkref_hworker, &jobs[t]) != 0) {
            vkref_hworker(&jobs[t]);
            tid[t] = 0;
        }
        used = t + 1;
    }
    for (int t = 0; t < used; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}
