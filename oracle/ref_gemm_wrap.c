/* ref_gemm_wrap.c -- compiles the reference's own CPU GEMM checker
 * (test/test_gemm.c of lakitu12/vkblas, included from the reference tree by
 * path at build time, never copied) into oracle/_ref/libvkref.so.
 *
 * TEST INFRASTRUCTURE ONLY: used to pin the oracle restatement and as the
 * "reference" CPU baseline.  The reference's main() is renamed and never
 * called; its device calls resolve to the failing stubs in stub_include/.
 */
#include <stdint.h>
#define main vkref_unused_test_gemm_main
#include REF_TEST_GEMM_C
#undef main

#define EXPORT __attribute__((visibility("default")))

/* test/test_gemm.c:32-58, called unmodified. transa/transb: 0 = N, 1 = T. */
EXPORT void vkref_ref_gemm(int transa, int transb, int m, int n, int k, float alpha,
                           const float* A, int lda, const float* B, int ldb, float beta,
                           float* C, int ldc, int sample_rows) {
    ref_gemm(transa ? HIPBLAS_OP_T : HIPBLAS_OP_N, transb ? HIPBLAS_OP_T : HIPBLAS_OP_N,
             m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, sample_rows);
}

/* All-core timing harness: rows [r0, r0+nr) of column-major C are split into
 * contiguous blocks and each pthread calls the unmodified ref_gemm on its
 * block (A offset i0 for op N, i0*lda for op T; C offset i0). */
#include <pthread.h>
struct vkref_job {
    int transa, transb, n, k, lda, ldb, ldc, i0, cnt;
    float alpha, beta;
    const float *A, *B;
    float* C;
};
static void* vkref_worker(void* p) {
    struct vkref_job* j = (struct vkref_job*)p;
    const float* Ab = j->transa ? j->A + (size_t)j->i0 * j->lda : j->A + j->i0;
    ref_gemm(j->transa ? HIPBLAS_OP_T : HIPBLAS_OP_N, j->transb ? HIPBLAS_OP_T : HIPBLAS_OP_N,
             j->cnt, j->n, j->k, j->alpha, Ab, j->lda, j->B, j->ldb, j->beta, j->C + j->i0,
             j->ldc, 0);
    return NULL;
}
EXPORT void vkref_ref_gemm_rows_mt(int transa, int transb, int m, int n, int k, float alpha,
                                   const float* A, int lda, const float* B, int ldb, float beta,
                                   float* C, int ldc, int r0, int nr, int threads) {
    (void)m;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    struct vkref_job jobs[256];
    pthread_t tid[256];
    int per = (nr + threads - 1) / threads, used = 0;
    for (int t = 0; t < threads; t++) {
        int cnt = nr - t * per;
        if (cnt > per) cnt = per;
        if (cnt <= 0) break;
        jobs[t] = (struct vkref_job){transa, transb, n, k, lda, ldb, ldc, r0 + t * per, cnt,
                                     alpha, beta, A, B, C};
        if (pthread_create(&tid[t], NULL, vkref_worker, &jobs[t]) != 0) {
            vkref_worker(&jobs[t]);
            tid[t] = 0;
        }
        used = t + 1;
    }
    for (int t = 0; t < used; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}
