/* Minimal stand-in for <hip/hip_runtime_api.h>, used ONLY to compile the
 * reference's CPU checkers into oracle/_ref/.  Every device call fails: the
 * wrapper translation units never call the reference's main(), they only
 * export its host-side reference GEMMs and half-precision converters. */
#pragma once
#include <stddef.h>

typedef int hipError_t;
typedef enum { hipMemcpyHostToDevice = 1, hipMemcpyDeviceToHost = 2 } hipMemcpyKind;
static inline hipError_t hipMalloc(void** p, size_t n) { (void)n; *p = 0; return 1; }
static inline hipError_t hipFree(void* p) { (void)p; return 1; }
static inline hipError_t hipMemcpy(void* d, const void* s, size_t n, hipMemcpyKind k) {
    (void)d; (void)s; (void)n; (void)k; return 1;
}
static inline hipError_t hipMemset(void* d, int v, size_t n) { (void)d; (void)v; (void)n; return 1; }
static inline hipError_t hipInit(unsigned f) { (void)f; return 1; }
static inline hipError_t hipSetDevice(int d) { (void)d; return 1; }
static inline hipError_t hipDeviceSynchronize(void) { return 1; }
