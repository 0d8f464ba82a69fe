"""ctypes signatures of the hipBLAS / rocBLAS ABI exported by libvkblas_hipblas.so.

A Python caller of the shim sees exactly what a C caller that dlopens the
library sees (the reference's tests bind it the same way:
test/test_gemm.c:14-22, 210-219; test/test_v9h.c:12-16).  Device pointers
are plain integers (e.g. ``tensor.data_ptr()``), scalars are passed by
pointer as hipBLAS requires.
"""
from __future__ import annotations

import ctypes as C

from . import lib

i32, i64, vp, u32 = C.c_int, C.c_longlong, C.c_void_p, C.c_uint32

_SIGS = {
    "hipblasCreate": [C.POINTER(vp)],
    "hipblasDestroy": [vp],
    "hipblasSetStream": [vp, vp],
    "hipblasGetStream": [vp, C.POINTER(vp)],
    "hipblasSetPointerMode": [vp, i32],
    "hipblasGetPointerMode": [vp, C.POINTER(i32)],
    "hipblasSetAtomicsMode": [vp, i32],
    "hipblasSetWorkspace": [vp, vp, C.c_size_t],
    "hipblasGetVersion": [vp, C.POINTER(i32)],
    "hipblasSgemm": [vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32],
    "hipblasSgemmStridedBatched": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i64, vp, i32, i64,
                                   vp, vp, i32, i64, i32],
    "hipblasGemmEx_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, i32, i32, vp, vp, i32,
                         i32, i32, i32],
    "hipblasGemmStridedBatchedEx_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, i64, vp, i32,
                                       i32, i64, vp, vp, i32, i32, i64, i32, i32, i32],
    "hipblasGemmEx": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, i32, i32, vp, vp, i32,
                      i32, i32, i32],
    "hipblasDgemm": [vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32],
    "hipblasDgemmStridedBatched": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i64, vp, i32, i64,
                                   vp, vp, i32, i64, i32],
    "hipblasCgemm_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32],
    "hipblasCgemmStridedBatched_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i64, vp, i32, i64,
                                      vp, vp, i32, i64, i32],
    "hipblasZgemm_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, vp, i32, vp, vp, i32],
    "hipblasZgemmStridedBatched_v2": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i64, vp, i32, i64,
                                      vp, vp, i32, i64, i32],
    "hipblasSdot": [vp, i32, vp, i32, vp, i32, vp],
    "rocblas_create_handle": [C.POINTER(vp)],
    "rocblas_destroy_handle": [vp],
    "rocblas_set_stream": [vp, vp],
    "rocblas_set_pointer_mode": [vp, i32],
    "rocblas_gemm_ex": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp, i32, i32, vp, vp, i32,
                        i32, vp, i32, i32, i32, i32, C.c_int32, C.c_uint32],
    "rocblas_gemm_strided_batched_ex": [vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, i64, vp, i32,
                                        i32, i64, vp, vp, i32, i32, i64, vp, i32, i32, i64, i32,
                                        i32, i32, C.c_int32, C.c_uint32],
}

for _name, _args in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = i32
lib.hipblasStatusToString.argtypes = [i32]
lib.hipblasStatusToString.restype = C.c_char_p


def fptr(x: float) -> C.Array:
    """A host fp32 scalar that lives as long as the returned object."""
    return (C.c_float * 1)(x)


class Handle:
    """RAII wrapper around a hipBLAS handle of the shim."""

    def __init__(self):
        self.h = vp()
        st = lib.hipblasCreate(C.byref(self.h))
        if st != 0:
            raise RuntimeError(f"hipblasCreate -> {st}")

    def set_stream(self, stream) -> int:
        if stream is not None and hasattr(stream, "cuda_stream"):
            stream = stream.cuda_stream
        return lib.hipblasSetStream(self.h, vp(stream or 0))

    def close(self) -> None:
        if self.h:
            lib.hipblasDestroy(self.h)
            self.h = vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class RocHandle:
    def __init__(self):
        self.h = vp()
        st = lib.rocblas_create_handle(C.byref(self.h))
        if st != 0:
            raise RuntimeError(f"rocblas_create_handle -> {st}")

    def set_stream(self, stream) -> int:
        if stream is not None and hasattr(stream, "cuda_stream"):
            stream = stream.cuda_stream
        return lib.rocblas_set_stream(self.h, vp(stream or 0))

    def close(self) -> None:
        if self.h:
            lib.rocblas_destroy_handle(self.h)
            self.h = vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
