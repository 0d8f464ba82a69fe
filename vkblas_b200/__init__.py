"""vkblas_b200 -- B200-native BLAS core behind the vkblas / hipBLAS C ABI.

The product is the shared library ``libvkblas_hipblas.so`` built in-tree from
``csrc/`` (see ``build.py``).  This package only loads it with ctypes and
offers thin helpers that pass torch tensors' device pointers to the C entry
points; no arithmetic happens in Python and there is no CPU fallback: if the
library is missing, importing raises.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libvkblas_hipblas.so")

VKBLAS_OK, VKBLAS_ERR_INIT, VKBLAS_ERR_IMPORT, VKBLAS_ERR_PARAM, VKBLAS_ERR_FALLBACK = range(5)
OP_N, OP_T = 0, 1
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
PATH_AUTO, PATH_SIMT, PATH_TC, PATH_GEMV = 0, 1, 2, 3
PATH_NAMES = {PATH_AUTO: "auto", PATH_SIMT: "simt", PATH_TC: "tc", PATH_GEMV: "gemv"}

# hipBLAS / rocBLAS ABI values (include/vkblas_hipblas.h)
HIPBLAS_OP_N, HIPBLAS_OP_T, HIPBLAS_OP_C = 111, 112, 113
HIPBLAS_STATUS_SUCCESS, HIPBLAS_STATUS_INVALID_VALUE, HIPBLAS_STATUS_NOT_SUPPORTED = 0, 3, 7
HIPBLAS_POINTER_MODE_HOST, HIPBLAS_POINTER_MODE_DEVICE = 0, 1
HIP_R_32F, HIP_R_16F, HIP_R_16BF = 0, 2, 14
HIPBLAS_R_16F, HIPBLAS_R_32F, HIPBLAS_R_16B = 150, 151, 168
HIPBLAS_COMPUTE_32F, HIPBLAS_COMPUTE_32F_PEDANTIC = 2, 3
HIPBLAS_GEMM_DEFAULT = 160
ROCBLAS_OP_N, ROCBLAS_OP_T = 111, 112
ROCBLAS_F16, ROCBLAS_F32, ROCBLAS_BF16 = 150, 151, 168
rocblas_status_success, rocblas_status_not_implemented, rocblas_status_invalid_value = 0, 2, 11


class VkblasError(RuntimeError):
    pass


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise VkblasError(
            f"{LIB_PATH} is missing: build it with `python -m vkblas_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    u32, i64, f32, vp, i32 = C.c_uint32, C.c_int64, C.c_float, C.c_void_p, C.c_int
    gemm_args = [i32, i32, u32, u32, u32, f32, vp, u32, vp, u32, f32, vp, u32, u32, i64, i64, i64]
    for name in ("vkblas_gemm_f32", "vkblas_gemm_f16", "vkblas_gemm_bf16", "vkblas_gemm_bf16_hipblas"):
        fn = getattr(lib, name)
        fn.argtypes = gemm_args
        fn.restype = i32
    lib.vkblas_gemm_ex.argtypes = [i32, i32, i32, u32, u32, u32, vp, vp, i32, vp, u32, vp, u32, vp,
                                   u32, u32, i64, i64, i64, vp]
    lib.vkblas_gemm_ex.restype = i32
    lib.vkblas_b200_gemm_replicated.argtypes = [i32, i32, i32, u32, u32, u32, f32, vp, u32, vp,
                                                u32, f32, vp, u32, u32, i64, i64, i64,
                                                C.POINTER(vp), u32, vp]
    lib.vkblas_b200_gemm_replicated.restype = i32
    lib.vkblas_gemv_splitk_noalloc.argtypes = [i32, u32, u32, u32, f32, vp, u32, vp, u32, f32, vp,
                                               u32, u32, vp]
    lib.vkblas_gemv_splitk_noalloc.restype = i32
    f64 = C.c_double
    lib.vkblas_gemm_f64.argtypes = [i32, i32, u32, u32, u32, f64, vp, u32, vp, u32, f64, vp, u32,
                                    u32, i64, i64, i64]
    lib.vkblas_gemm_c64.argtypes = [i32, i32, u32, u32, u32, f32, f32, vp, u32, vp, u32, f32, f32,
                                    vp, u32, u32, i64, i64, i64]
    lib.vkblas_gemm_z64.argtypes = [i32, i32, u32, u32, u32, f64, f64, vp, u32, vp, u32, f64, f64,
                                    vp, u32, u32, i64, i64, i64]
    for name in ("vkblas_gemm_f64", "vkblas_gemm_c64", "vkblas_gemm_z64"):
        getattr(lib, name).restype = i32
    lib.vkblas_set_stream.argtypes = [vp]
    lib.vkblas_get_stream.restype = vp
    lib.vkblas_b200_set_path.argtypes = [i32]
    lib.vkblas_b200_get_path.restype = i32
    lib.vkblas_b200_last_path.restype = i32
    lib.vkblas_b200_last_split.restype = i32
    lib.vkblas_b200_last_pair.restype = i32
    lib.vkblas_b200_last_tile_n.restype = i32
    lib.vkblas_b200_set_splitk.argtypes = [i32]
    lib.vkblas_b200_set_test_stall.argtypes = [i32]
    lib.vkblas_b200_set_test_alloc_fail.argtypes = [i32]
    lib.vkblas_b200_device_status.argtypes = [i32]
    lib.vkblas_b200_device_status.restype = i32
    lib.vkblas_b200_launch_count.restype = C.c_uint64
    lib.vkblas_b200_set_kernel_events.argtypes = [vp, vp]
    lib.vkblas_b200_release_workspaces.argtypes = [vp, i32]
    lib.vkblas_b200_release_workspaces.restype = i32
    lib.vkblas_b200_version.restype = C.c_char_p
    lib.vkblas_cache_invalidate_base.argtypes = [vp]
    lib.vkblas_shard_range.argtypes = [C.c_uint64, C.c_uint64, i32, i32,
                                       C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
    lib.vkblas_shard_range.restype = i32
    lib.vkblas_b200_tc_plan.argtypes = [i32, i32, i32, u32, u32, u32, u32, i32, i32, vp]
    lib.vkblas_b200_tc_plan.restype = i32
    lib.vkblas_b200_peak_launch.argtypes = [i32, u32, vp, vp, C.POINTER(C.c_double)]
    lib.vkblas_b200_peak_launch.restype = i32
    return lib


_lib = None


def _get() -> C.CDLL:
    """The loaded library (loaded on first use, so that building it does not need it)."""
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def __getattr__(name):
    if name == "lib":
        return _get()
    raise AttributeError(name)


def version() -> str:
    return _get().vkblas_b200_version().decode()


def set_stream(stream) -> None:
    """Stream (cudaStream_t as int, or a torch.cuda.Stream) for this thread's calls."""
    if stream is not None and hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    _get().vkblas_set_stream(C.c_void_p(stream or 0))


def set_path(path: int) -> None:
    _get().vkblas_b200_set_path(int(path))


def last_path() -> int:
    return _get().vkblas_b200_last_path()


def last_split() -> int:
    """K-split count of this thread's last call (1 = none)."""
    return _get().vkblas_b200_last_split()


def last_pair() -> bool:
    """Whether this thread's last call ran on 2-CTA clusters (256-row tiles)."""
    return bool(_get().vkblas_b200_last_pair())


def last_tile_n() -> int:
    """N width of the tensor-core tile of this thread's last call (0: not tensor-core)."""
    return _get().vkblas_b200_last_tile_n()


def set_splitk(s: int) -> None:
    _get().vkblas_b200_set_splitk(int(s))


def device_status(clear: bool = True) -> int:
    return _get().vkblas_b200_device_status(1 if clear else 0)


def set_kernel_events(start=None, end=None) -> None:
    """Record torch.cuda.Event `start`/`end` around the main kernel of each
    following call on this thread (None, None: off).  The events must have
    been recorded once already, so that their CUDA handles exist."""
    def handle(e):
        if e is None:
            return None
        h = e.cuda_event
        if not h:
            raise VkblasError("record the event once before passing it")
        return h
    _get().vkblas_b200_set_kernel_events(handle(start), handle(end))


def release_workspaces(stream=None, all_streams: bool = False) -> None:
    """Free the library's scratch for `stream` (a torch.cuda.Stream, a raw
    handle or None = default stream), or for every stream; synchronises the device."""
    if stream is not None and hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    if _get().vkblas_b200_release_workspaces(stream, 1 if all_streams else 0) != 0:
        raise VkblasError("vkblas_b200_release_workspaces failed")


def launch_count() -> int:
    return int(_get().vkblas_b200_launch_count())


class _TcPlan(C.Structure):
    _fields_ = [(name, C.c_uint32) for name in (
        "tile_m", "tile_n", "transposed", "pair", "tiles", "full_tiles", "splits", "kblocks",
        "kblocks_per_split")] + [("partial_bytes", C.c_uint64), ("tail_tiles", C.c_uint32)]


def tc_plan(dtype: int, op_a: int, op_b: int, M: int, N: int, K: int, batch: int = 1,
            num_sms: int = 148, allow_wide: bool = True) -> dict:
    """Tile and split plan of a tensor-core GEMM (vkblas_b200_tc_plan; pure
    host logic, no GPU needed) as a dict of the struct's fields."""
    out = _TcPlan()
    st = _get().vkblas_b200_tc_plan(dtype, op_a, op_b, M, N, K, batch, num_sms,
                                    1 if allow_wide else 0, C.byref(out))
    if st != VKBLAS_OK:
        raise VkblasError(f"vkblas_b200_tc_plan status {st}")
    return {name: int(getattr(out, name)) for name, _ in _TcPlan._fields_}


def shard_range(units: int, rank: int, world: int, block: int = 1):
    b = C.c_uint64()
    n = C.c_uint64()
    st = _get().vkblas_shard_range(units, block, rank, world, C.byref(b), C.byref(n))
    if st != VKBLAS_OK:
        raise VkblasError(f"vkblas_shard_range status {st}")
    return int(b.value), int(n.value)


_GEMM_BY_DTYPE = {DT_F32: "vkblas_gemm_f32", DT_F16: "vkblas_gemm_f16", DT_BF16: "vkblas_gemm_bf16"}


def gemm(dtype: int, op_a: int, op_b: int, M: int, N: int, K: int, alpha: float, A: int, lda: int,
         B: int, ldb: int, beta: float, C_: int, ldc: int, batch: int = 1, sa: int = 0,
         sb: int = 0, sc: int = 0) -> int:
    """Row-major engine call (reference src/vkblas.h:19-36) on raw device pointers.

    Returns the vkblas_status_t value."""
    fn = getattr(_get(), _GEMM_BY_DTYPE[dtype])
    return fn(op_a, op_b, M, N, K, alpha, A, lda, B, ldb, beta, C_, ldc, batch, sa, sb, sc)


def gemm_replicated(dtype: int, op_a: int, op_b: int, M: int, N: int, K: int, alpha: float,
                    A: int, lda: int, B: int, ldb: int, beta: float, C_: int, ldc: int,
                    peers, batch: int = 1, sa: int = 0, sb: int = 0, sc: int = 0,
                    stream=None) -> int:
    """vkblas_b200_gemm_replicated on raw device pointers: the engine call,
    with every C element also stored at the same offset from each address in
    ``peers`` (at most 7).  ``stream``: a torch stream, a raw cudaStream_t or
    None (legacy default stream).  Returns the vkblas_status_t value."""
    arr = (C.c_void_p * max(1, len(peers)))(*[C.c_void_p(int(x)) for x in peers])
    raw = getattr(stream, "cuda_stream", stream)
    return _get().vkblas_b200_gemm_replicated(dtype, op_a, op_b, M, N, K, alpha, A, lda, B, ldb,
                                              beta, C_, ldc, batch, sa, sb, sc, arr, len(peers),
                                              raw)


def dtype_of(t) -> int:
    import torch
    return {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}[t.dtype]


def _extent(rows: int, cols: int, ld: int, batch: int, stride: int) -> int:
    """Elements a row-major operand addresses: the last batch entry's last row
    ends at (batch - 1) * stride + (rows - 1) * ld + cols."""
    return (batch - 1) * stride + (rows - 1) * ld + cols


def _check_tensors(op_a, op_b, M, N, K, A, lda, B, ldb, Cout, ldc, batch, sa, sb, sc) -> None:
    """Host-side checks of gemm_tensors' operands, before anything is launched:
    CUDA tensors of one dtype on one device, contiguous (the engine addresses
    their flat storage), and large enough for the addressed extents."""
    ts = {"A": A, "B": B, "C": Cout}
    for name, t in ts.items():
        if not getattr(t, "is_cuda", False):
            raise ValueError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous (flat storage, element strides)")
    if not (A.dtype == B.dtype == Cout.dtype):
        raise ValueError(f"dtypes differ: {A.dtype}, {B.dtype}, {Cout.dtype}")
    if not (A.device == B.device == Cout.device):
        raise ValueError(f"devices differ: {A.device}, {B.device}, {Cout.device}")
    if min(M, N, K, batch) <= 0:
        raise ValueError("M, N, K and batch must be positive")
    ra, ca = (K, M) if op_a else (M, K)
    rb, cb = (N, K) if op_b else (K, N)
    for name, t, r, c, ld, st in (("A", A, ra, ca, lda, sa), ("B", B, rb, cb, ldb, sb),
                                  ("C", Cout, M, N, ldc, sc)):
        if ld < c:
            raise ValueError(f"ld{name.lower()} = {ld} < {c}")
        need = _extent(r, c, ld, batch, st)
        if t.numel() < need:
            raise ValueError(f"{name} holds {t.numel()} elements, the call addresses {need}")


def gemm_tensors(op_a: int, op_b: int, M: int, N: int, K: int, alpha: float, A, lda: int, B,
                 ldb: int, beta: float, Cout, ldc: int, batch: int = 1, sa: int = 0, sb: int = 0,
                 sc: int = 0, stream=None) -> None:
    """Engine call on torch CUDA tensors (flat storage, element strides), on
    ``stream`` (default: torch's current stream), on the tensors' device.
    Raises ValueError for operands that do not fit the call, VkblasError on a
    non-OK status."""
    import torch
    _check_tensors(op_a, op_b, M, N, K, A, lda, B, ldb, Cout, ldc, batch, sa, sb, sc)
    with torch.cuda.device(A.device):
        if stream is None:
            stream = torch.cuda.current_stream()
        set_stream(stream)
        st = gemm(dtype_of(A), op_a, op_b, M, N, K, alpha, A.data_ptr(), lda, B.data_ptr(), ldb,
                  beta, Cout.data_ptr(), ldc, batch, sa, sb, sc)
    if st != VKBLAS_OK:
        raise VkblasError(f"vkblas gemm returned status {st}")
