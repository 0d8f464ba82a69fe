"""ctypes front end of the CPU oracle (test infrastructure only).

Wraps ``liboracle.so`` (our C restatement of the reference arithmetic, see
``gemm_oracle.c``) and, when it was built, ``_ref/libvkref.so`` (the
reference's own CPU checkers test/test_gemm.c:32-58 and test/test_h.c:16-79,
compiled from the reference tree).  All arrays are numpy, C-contiguous.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(_HERE, "liboracle.so")
_REF_SO = os.path.join(_HERE, "_ref", "libvkref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i, _u32, _i64, _f, _d, _sz = C.c_int, C.c_uint32, C.c_int64, C.c_float, C.c_double, C.c_size_t


def build() -> None:
    """Compile liboracle.so (and _ref/libvkref.so when $VKBLAS_REFERENCE_DIR names
    the reference tree)."""
    ref = os.environ.get("VKBLAS_REFERENCE_DIR", "")
    subprocess.run(["make", "-s", "-C", _HERE, "REFERENCE_DIR=" + ref], check=True)


def _load():
    if not os.path.exists(_ORACLE_SO):
        build()
    lib = C.CDLL(_ORACLE_SO)
    lib.orc_f2h_rne.restype = C.c_uint16
    lib.orc_f2h_rne.argtypes = [_f]
    lib.orc_h2f.restype = _f
    lib.orc_h2f.argtypes = [C.c_uint16]
    lib.orc_f2bf_rne.restype = C.c_uint16
    lib.orc_f2bf_rne.argtypes = [_f]
    lib.orc_bf2f.restype = _f
    lib.orc_bf2f.argtypes = [C.c_uint16]
    lib.orc_f2h_test_h.restype = C.c_uint16
    lib.orc_f2h_test_h.argtypes = [_f]
    lib.orc_sgemm_colmajor_f64acc.argtypes = [_i, _i, _i, _i, _i, _f, _f32p, _i, _f32p, _i, _f, _f32p, _i]
    lib.orc_gemm_rowmajor_f32seq.argtypes = [_i, _i, _u32, _u32, _u32, _f, _f32p, _u32, _f32p, _u32,
                                             _f, _f32p, _u32, _u32, _i64, _i64, _i64]
    lib.orc_gemm_rowmajor_f64.argtypes = [_i, _i, _u32, _u32, _u32, _d, _f32p, _u32, _f32p, _u32,
                                          _d, C.c_void_p, _u32, _f64p, _u32, _i64, _i64, _i64]
    lib.orc_hgemm_rowmajor.argtypes = [_i, _i, _i, _i, _u32, _u32, _u32, _f, _u16p, _u32, _u16p, _u32,
                                       _f, _u16p, _u32, _u32, _i64, _i64, _i64]
    lib.orc_hgemm_rowmajor_splitk.argtypes = [_i, _i, _i, _u32, _u32, _u32, _u32, _f, _u16p, _u32,
                                              _u16p, _u32, _f, _u16p, _u32, _i]
    lib.orc_gemm_rowmajor_f32_splitk.argtypes = [_i, _i, _u32, _u32, _u32, _u32, _f, _f32p, _u32,
                                                 _f32p, _u32, _f, _f32p, _u32]
    lib.orc_dgemm_rowmajor_seq.argtypes = [_i, _i, _u32, _u32, _u32, _d, _f64p, _u32, _f64p, _u32,
                                           _d, _f64p, _u32, _u32, _i64, _i64, _i64]
    lib.orc_cgemm_rowmajor.argtypes = [_i, _i, _u32, _u32, _u32, _f, _f, _f32p, _u32, _f32p, _u32,
                                       _f, _f, _f32p, _u32, _u32, _i64, _i64, _i64]
    lib.orc_zgemm_rowmajor.argtypes = [_i, _i, _u32, _u32, _u32, _d, _d, _f64p, _u32, _f64p, _u32,
                                       _d, _d, _f64p, _u32, _u32, _i64, _i64, _i64]
    lib.orc_gen_test_gemm.argtypes = [C.c_uint, _f32p, _sz, _f32p, _sz, _f32p, _sz]
    lib.orc_gen_test_h.argtypes = [C.c_uint, _i, _u16p, _sz, _u16p, _sz, _u16p, _sz, _i]
    lib.orc_sgemm_colmajor_rows_mt.argtypes = [_i, _i, _i, _i, _i, _f, _f32p, _i, _f32p, _i, _f,
                                               _f32p, _i, _i, _i, _i]
    return lib


def _load_ref():
    if not os.path.exists(_REF_SO):
        return None
    lib = C.CDLL(_REF_SO)
    lib.vkref_ref_gemm.argtypes = [_i, _i, _i, _i, _i, _f, _f32p, _i, _f32p, _i, _f, _f32p, _i, _i]
    lib.vkref_ref_gemm_rows_mt.argtypes = [_i, _i, _i, _i, _i, _f, _f32p, _i, _f32p, _i, _f, _f32p,
                                           _i, _i, _i, _i]
    lib.vkref_cpu_ref_half.argtypes = [_i, _i, _i, _i, _i, _i, _u16p, _i, _u16p, _i, _f, _f, _u16p, _i]
    lib.vkref_cpu_ref_half_cols_mt.argtypes = [_i, _i, _i, _i, _i, _i, _u16p, _i, _u16p, _i, _f, _f,
                                               _u16p, _i, _i, _i, _i]
    lib.vkref_f2h.restype = C.c_uint16
    lib.vkref_f2h.argtypes = [_f]
    lib.vkref_h2f.restype = _f
    lib.vkref_h2f.argtypes = [C.c_uint16]
    lib.vkref_f2bf.restype = C.c_uint16
    lib.vkref_f2bf.argtypes = [_f]
    lib.vkref_bf2f.restype = _f
    lib.vkref_bf2f.argtypes = [C.c_uint16]
    return lib


lib = _load()
ref = _load_ref()   # None when the reference build is absent


# ------------------------------------------------------------------ converters
def f2h(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits, exact RNE (numpy's own conversion is also RNE)."""
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def h2f(h: np.ndarray) -> np.ndarray:
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


def f2bf(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, RNE (vectorised form of orc_f2bf_rne)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf2f(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def widen(dtype: int, bits: np.ndarray) -> np.ndarray:
    return bf2f(bits) if dtype else h2f(bits)


def narrow(dtype: int, x: np.ndarray) -> np.ndarray:
    return f2bf(x) if dtype else f2h(x)


# ------------------------------------------------------------------- GEMMs
def sgemm_colmajor_f64acc(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc):
    """ref_gemm semantics, in place on C (column-major, test/test_gemm.c:32-58)."""
    lib.orc_sgemm_colmajor_f64acc(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)


def gemm_rowmajor_f32seq(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                         batch=1, sa=0, sb=0, sc=0):
    """Engine contract, sequential-fmaf fp32 accumulation, in place on C."""
    lib.orc_gemm_rowmajor_f32seq(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                                 batch, sa, sb, sc)


def gemm_rowmajor_f64(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, Cin, ldc,
                      batch=1, sa=0, sb=0, sc=0) -> np.ndarray:
    """Double-precision result of the engine contract: (batch, M, N) float64."""
    out = np.zeros((batch, M, N), np.float64)
    cptr = Cin.ctypes.data if (Cin is not None and beta != 0.0) else None
    lib.orc_gemm_rowmajor_f64(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, cptr, ldc, out,
                              batch, sa, sb, sc)
    return out


def hgemm_rowmajor(dtype, acc_mode, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc,
                   batch=1, sa=0, sb=0, sc=0):
    """Half-precision engine contract, in place on C (uint16 bit patterns)."""
    lib.orc_hgemm_rowmajor(dtype, acc_mode, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C,
                           ldc, batch, sa, sb, sc)


def hgemm_rowmajor_f64(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, Cin, ldc,
                       batch=1, sa=0, sb=0, sc=0) -> np.ndarray:
    """Double-precision yardstick for 2-byte inputs: (batch, M, N) float64."""
    Af = widen(dtype, A).astype(np.float32)
    Bf = widen(dtype, B).astype(np.float32)
    Cf = widen(dtype, Cin).astype(np.float32) if Cin is not None else None
    return gemm_rowmajor_f64(op_a, op_b, M, N, K, alpha, np.ascontiguousarray(Af), lda,
                             np.ascontiguousarray(Bf), ldb, beta,
                             None if Cf is None else np.ascontiguousarray(Cf), ldc, batch, sa, sb, sc)


def hgemm_rowmajor_splitk(dtype, op_a, op_b, M, N, K, nseg, alpha, A, lda, B, ldb, beta, C, ldc,
                          rounding=0):
    """Segmented fp32 sums added in order, alpha/beta, then the store encoder:
    rounding 0 = RNE (this library), 1 = the reference reduce's encoders
    (bf16 truncated, splitk_reduce_half.comp:8)."""
    lib.orc_hgemm_rowmajor_splitk(dtype, op_a, op_b, M, N, K, nseg, alpha, A, lda, B, ldb, beta, C, ldc,
                                  rounding)


def gemm_rowmajor_f32_splitk(op_a, op_b, M, N, K, span, alpha, A, lda, B, ldb, beta, C, ldc):
    """fp32 split-K model: segments of `span` k, each a sequential fmaf sum,
    added in segment order, then the fp32 epilogue (C updated in place)."""
    lib.orc_gemm_rowmajor_f32_splitk(op_a, op_b, M, N, K, span, alpha, A, lda, B, ldb, beta, C, ldc)


def dgemm_rowmajor_seq(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch=1,
                       sa=0, sb=0, sc=0):
    """fp64 engine contract, sequential fma; C (float64) updated in place."""
    lib.orc_dgemm_rowmajor_seq(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch,
                               sa, sb, sc)


def cgemm_rowmajor(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch=1, sa=0, sb=0,
                   sc=0):
    """complex64 the reference's way (interleaved float32 arrays, C in place)."""
    lib.orc_cgemm_rowmajor(op_a, op_b, M, N, K, alpha.real, alpha.imag, A, lda, B, ldb, beta.real,
                           beta.imag, C, ldc, batch, sa, sb, sc)


def zgemm_rowmajor(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, batch=1, sa=0, sb=0,
                   sc=0):
    """complex128 the reference's way (interleaved float64 arrays, C in place)."""
    lib.orc_zgemm_rowmajor(op_a, op_b, M, N, K, alpha.real, alpha.imag, A, lda, B, ldb, beta.real,
                           beta.imag, C, ldc, batch, sa, sb, sc)


# -------------------------------------------------------------- generators
def gen_test_gemm(seed: int, na: int, nb: int, nc: int):
    """Inputs exactly as test/test_gemm.c:70-73 builds them (glibc rand)."""
    A = np.empty(na, np.float32)
    B = np.empty(nb, np.float32)
    Cc = np.empty(nc, np.float32)
    lib.orc_gen_test_gemm(seed, A, na, B, nb, Cc, nc)
    return A, B, Cc


def gen_test_h(seed: int, dtype: int, na: int, nb: int, nc: int, batched: bool):
    """Inputs exactly as test/test_h.c:102-118 / 170-186 builds them."""
    A = np.empty(na, np.uint16)
    B = np.empty(nb, np.uint16)
    Cc = np.empty(nc, np.uint16)
    lib.orc_gen_test_h(seed, dtype, A, na, B, nb, Cc, nc, 1 if batched else 0)
    return A, B, Cc


# ---------------------------------------------------------- error measures
def rel_frobenius(got: np.ndarray, want: np.ndarray) -> float:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.linalg.norm(want.ravel())
    num = np.linalg.norm((got - want).ravel())
    return float(num / den) if den > 0 else float(num)
