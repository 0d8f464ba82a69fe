/* A stand-in "real" cuBLAS for the interposer's forwarding tests (host only).
 * Its handles are the constant 0xC0B1; every GEMM records which entry point it
 * was and the arguments that matter, so a test can check that a declined call
 * reached the real library unchanged. */
#include <stdint.h>

#define FAKE_HANDLE ((void*)0xC0B1)

int fake_last = 0;          /* 1 Sgemm_v2, 2 SgemmStridedBatched, 3 SgemmEx, 4 GemmEx,
                               5 GemmStridedBatchedEx, 6 Hgemm, 7 HgemmStridedBatched */
long long fake_args[12];    /* m, n, k, lda, ldb, ldc, type/batch, compute, algo, strideC, ... */
const void* fake_alpha = 0;

static int mark(void* h, int which, int m, int n, int k, int lda, int ldb, int ldc, const void* al) {
    fake_last = which;
    fake_args[0] = m; fake_args[1] = n; fake_args[2] = k;
    fake_args[3] = lda; fake_args[4] = ldb; fake_args[5] = ldc;
    fake_alpha = al;
    return h == FAKE_HANDLE ? 0 : 1;
}

int cublasGetStream_v2(void* h, void** s) { *s = 0; return h == FAKE_HANDLE ? 0 : 1; }
int cublasGetPointerMode_v2(void* h, int* m) { *m = 0; return h == FAKE_HANDLE ? 0 : 1; }
int cublasGetMathMode(void* h, int* m) { *m = 0; return h == FAKE_HANDLE ? 0 : 1; }

int cublasSgemm_v2(void* h, int ta, int tb, int m, int n, int k, const float* al, const float* A,
                   int lda, const float* B, int ldb, const float* be, float* C, int ldc) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C;
    return mark(h, 1, m, n, k, lda, ldb, ldc, al);
}
int cublasSgemmStridedBatched(void* h, int ta, int tb, int m, int n, int k, const float* al,
                              const float* A, int lda, long long sA, const float* B, int ldb,
                              long long sB, const float* be, float* C, int ldc, long long sC,
                              int batch) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C; (void)sA; (void)sB;
    fake_args[6] = batch; fake_args[9] = sC;
    return mark(h, 2, m, n, k, lda, ldb, ldc, al);
}
int cublasSgemmEx(void* h, int ta, int tb, int m, int n, int k, const float* al, const void* A,
                  int at, int lda, const void* B, int bt, int ldb, const float* be, void* C, int ct,
                  int ldc) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C; (void)bt;
    fake_args[6] = at * 100 + ct;
    int r = mark(h, 3, m, n, k, lda, ldb, ldc, al);
    fake_args[6] = at * 100 + ct;
    return r;
}
int cublasGemmEx(void* h, int ta, int tb, int m, int n, int k, const void* al, const void* A,
                 int at, int lda, const void* B, int bt, int ldb, const void* be, void* C, int ct,
                 int ldc, int compute, int algo) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C; (void)bt;
    int r = mark(h, 4, m, n, k, lda, ldb, ldc, al);
    fake_args[6] = at * 100 + ct; fake_args[7] = compute; fake_args[8] = algo;
    return r;
}
int cublasGemmStridedBatchedEx(void* h, int ta, int tb, int m, int n, int k, const void* al,
                               const void* A, int at, int lda, long long sA, const void* B, int bt,
                               int ldb, long long sB, const void* be, void* C, int ct, int ldc,
                               long long sC, int batch, int compute, int algo) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C; (void)bt; (void)sA; (void)sB; (void)at;
    (void)ct;
    int r = mark(h, 5, m, n, k, lda, ldb, ldc, al);
    fake_args[6] = batch; fake_args[7] = compute; fake_args[8] = algo; fake_args[9] = sC;
    return r;
}
int cublasHgemm(void* h, int ta, int tb, int m, int n, int k, const void* al, const void* A,
                int lda, const void* B, int ldb, const void* be, void* C, int ldc) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C;
    return mark(h, 6, m, n, k, lda, ldb, ldc, al);
}
int cublasHgemmStridedBatched(void* h, int ta, int tb, int m, int n, int k, const void* al,
                              const void* A, int lda, long long sA, const void* B, int ldb,
                              long long sB, const void* be, void* C, int ldc, long long sC,
                              int batch) {
    (void)ta; (void)tb; (void)A; (void)B; (void)be; (void)C; (void)sA; (void)sB;
    int r = mark(h, 7, m, n, k, lda, ldb, ldc, al);
    fake_args[6] = batch; fake_args[9] = sC;
    return r;
}
