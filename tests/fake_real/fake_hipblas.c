/* A stand-in "real" hipBLAS/rocBLAS for the forwarding tests (host only).
 * Its handles are the constant 0x5EA1; each forwarded call checks that it was
 * given that handle (i.e. that the shim unwrapped its own) and leaves a mark. */
#include <stdint.h>
#include <stddef.h>

#define FAKE_HANDLE ((void*)0x5EA1)
int fake_last_call = 0;          /* 1 sdot, 2 sgemm, 3 dgemm, 4 setstream, 5 rocblas_gemm_ex,
                                    6 rocblas_gemm_strided_batched_ex */
long long fake_last_strides[4];  /* strideA, strideB, strideC, strideD of the last call 6 */

int hipblasCreate(void** h) { *h = FAKE_HANDLE; return 0; }
int hipblasDestroy(void* h) { return h == FAKE_HANDLE ? 0 : 3; }
int hipblasSetStream(void* h, void* s) { (void)s; fake_last_call = 4; return h == FAKE_HANDLE ? 0 : 3; }
int hipblasSetPointerMode(void* h, int m) { (void)m; return h == FAKE_HANDLE ? 0 : 3; }
int hipblasGetVersion(void* h, int* v) { *v = 424242; return h == FAKE_HANDLE ? 0 : 3; }
const char* hipblasStatusToString(int s) { (void)s; return "fake-status"; }
int hipblasSdot(void* h, int n, const float* x, int incx, const float* y, int incy, float* r) {
    (void)n; (void)x; (void)incx; (void)y; (void)incy;
    fake_last_call = 1;
    if (h != FAKE_HANDLE) return 3;
    *r = 42.0f;
    return 0;
}
int hipblasSgemm(void* h, int ta, int tb, int m, int n, int k, const float* al, const float* A,
                 int lda, const float* B, int ldb, const float* be, float* C, int ldc) {
    (void)ta; (void)tb; (void)m; (void)n; (void)k; (void)al; (void)A; (void)lda; (void)B;
    (void)ldb; (void)be; (void)C; (void)ldc;
    fake_last_call = 2;
    return h == FAKE_HANDLE ? 0 : 3;
}
int hipblasDgemm(void* h, int ta, int tb, int m, int n, int k, const double* al, const double* A,
                 int lda, const double* B, int ldb, const double* be, double* C, int ldc) {
    (void)ta; (void)tb; (void)m; (void)n; (void)k; (void)al; (void)A; (void)lda; (void)B;
    (void)ldb; (void)be; (void)C; (void)ldc;
    fake_last_call = 3;
    return h == FAKE_HANDLE ? 0 : 3;
}
int rocblas_create_handle(void** h) { *h = FAKE_HANDLE; return 0; }
int rocblas_destroy_handle(void* h) { return h == FAKE_HANDLE ? 0 : 1; }
int rocblas_gemm_ex(void* h, int ta, int tb, int m, int n, int k, const void* al, const void* a,
                    int at, int lda, const void* b, int bt, int ldb, const void* be, const void* c,
                    int ct, int ldc, void* d, int dt, int ldd, int comp, int algo, int32_t sol,
                    uint32_t flags) {
    (void)ta; (void)tb; (void)m; (void)n; (void)k; (void)al; (void)a; (void)at; (void)lda;
    (void)b; (void)bt; (void)ldb; (void)be; (void)c; (void)ct; (void)ldc; (void)d; (void)dt;
    (void)ldd; (void)comp; (void)algo; (void)sol; (void)flags;
    fake_last_call = 5;
    return h == FAKE_HANDLE ? 0 : 1;
}
int rocblas_gemm_strided_batched_ex(void* h, int ta, int tb, int m, int n, int k, const void* al,
                                    const void* a, int at, int lda, long long sa, const void* b,
                                    int bt, int ldb, long long sb, const void* be, const void* c,
                                    int ct, int ldc, long long sc, void* d, int dt, int ldd,
                                    long long sd, int batch, int comp, int algo, int32_t sol,
                                    uint32_t flags) {
    (void)ta; (void)tb; (void)m; (void)n; (void)k; (void)al; (void)a; (void)at; (void)lda;
    (void)b; (void)bt; (void)ldb; (void)be; (void)c; (void)ct; (void)ldc; (void)d; (void)dt;
    (void)ldd; (void)batch; (void)comp; (void)algo; (void)sol; (void)flags;
    fake_last_call = 6;
    fake_last_strides[0] = sa; fake_last_strides[1] = sb;
    fake_last_strides[2] = sc; fake_last_strides[3] = sd;
    return h == FAKE_HANDLE ? 0 : 1;
}
long long fake_get_last_stride(int i) { return fake_last_strides[i]; }
int fake_get_last_call(void) { return fake_last_call; }
