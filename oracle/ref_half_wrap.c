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
