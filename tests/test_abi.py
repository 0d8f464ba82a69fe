"""C-ABI boundary tests that need no GPU.

* libvkblas_hipblas.so loads and exports every function include/*.h declares
  (and nothing from the CUDA runtime it links statically);
* host-side behaviour of the hipBLAS/rocBLAS shim: handle state, argument
  validation before any device work (src/vkblas_hipblas.c:223, 406),
  forwarding of unhandled calls to the real library with the real handle,
  NOT_SUPPORTED / not_implemented when no real library exists
  (src/vkblas_hipblas.c:62-65, 821-824);
* engine argument validation and the "no usable device" status;
* the multi-GPU shard planner.
"""
import ctypes as C
import os
import re
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import hipblas as hb  # noqa: E402


def _declared_functions(headers=None):
    names = set()
    for f in os.listdir(INCLUDE):
        if not f.endswith(".h"):
            continue
        if headers is None and f == "vkblas_cublas.h":    # declares libvkblas_cublas.so's API
            continue
        if headers is not None and f not in headers:
            continue
        text = open(os.path.join(INCLUDE, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"typedef[^;]*;", "", text, flags=re.S)
        for m in re.finditer(r"(?:^|\n)\s*(?:const\s+)?[A-Za-z_]\w*[\s\*]+([A-Za-z_]\w*)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", vk.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_every_declared_symbol_is_exported():
    decl = _declared_functions()
    assert len(decl) > 70
    exp = _exported()
    missing = [d for d in decl if d not in exp]
    assert not missing, missing
    for name in decl:
        getattr(vk.lib, name)        # dlsym through ctypes


def test_no_cuda_runtime_symbols_leak():
    leaked = [s for s in _exported() if s.startswith(("cuda", "__cuda", "cu"))]
    assert not leaked, leaked[:10]


def test_version():
    assert "sm_100a" in vk.version()


def test_hipblas_handle_state():
    with hb.Handle() as h:
        mode = C.c_int(-1)
        assert vk.lib.hipblasGetPointerMode(h.h, C.byref(mode)) == 0 and mode.value == 0
        assert vk.lib.hipblasSetPointerMode(h.h, 1) == 0
        assert vk.lib.hipblasGetPointerMode(h.h, C.byref(mode)) == 0 and mode.value == 1
        assert vk.lib.hipblasSetPointerMode(h.h, 7) == vk.HIPBLAS_STATUS_INVALID_VALUE
        assert vk.lib.hipblasSetStream(h.h, C.c_void_p(0x1234)) == 0
        s = C.c_void_p()
        assert vk.lib.hipblasGetStream(h.h, C.byref(s)) == 0 and s.value == 0x1234
        assert vk.lib.hipblasSetWorkspace(h.h, None, 0) == 0
        assert vk.lib.hipblasSetAtomicsMode(h.h, 1) == 0
        v = C.c_int()
        assert vk.lib.hipblasGetVersion(h.h, C.byref(v)) == 0 and v.value > 0
    assert vk.lib.hipblasStatusToString(3) == b"HIPBLAS_STATUS_INVALID_VALUE"


def test_hipblas_argument_validation_before_device_work():
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    # NULL handle (src/vkblas_hipblas.c:406)
    assert vk.lib.hipblasSgemm(None, 111, 111, 4, 4, 4, al, 0, 4, 0, 4, be, 0, 4) == 3
    with hb.Handle() as h:
        # m, n, k <= 0 (src/vkblas_hipblas.c:223)
        for m, n, k in ((0, 4, 4), (4, 0, 4), (4, 4, 0), (-1, 4, 4)):
            assert vk.lib.hipblasSgemm(h.h, 111, 111, m, n, k, al, 0, 4, 0, 4, be, 0, 4) == 3
        assert vk.lib.hipblasSgemmStridedBatched(h.h, 111, 111, 4, 4, 4, al, 0, 4, 16, 0, 4, 16,
                                                 be, 0, 4, 16, 0) == 3
        assert vk.lib.hipblasGemmEx_v2(h.h, 111, 111, 0, 4, 4, al, 0, vk.HIP_R_16F, 4, 0,
                                       vk.HIP_R_16F, 4, be, 0, vk.HIP_R_16F, 4, 2, 160) == 3
        assert vk.lib.hipblasDgemm(h.h, 111, 111, 0, 4, 4, None, 0, 4, 0, 4, None, 0, 4) == 3


def test_unhandled_calls_report_not_supported_without_real_library():
    with hb.Handle() as h:
        r = C.c_float(0)
        assert vk.lib.hipblasSdot(h.h, 4, 0, 1, 0, 1, C.byref(r)) == vk.HIPBLAS_STATUS_NOT_SUPPORTED
        al = (C.c_double * 1)(1.0)
        assert vk.lib.hipblasDgemm(h.h, 111, 111, 4, 4, 4, al, 0, 4, 0, 4, al, 0, 4) == \
            vk.HIPBLAS_STATUS_NOT_SUPPORTED
        # fp32 through the legacy hipblasGemmEx is forwarded (src/vkblas_hipblas.c:454-466)
        a1, b0 = hb.fptr(1.0), hb.fptr(0.0)
        assert vk.lib.hipblasGemmEx(h.h, 111, 111, 4, 4, 4, a1, 0, vk.HIPBLAS_R_32F, 4, 0,
                                    vk.HIPBLAS_R_32F, 4, b0, 0, vk.HIPBLAS_R_32F, 4, 151, 160) == \
            vk.HIPBLAS_STATUS_NOT_SUPPORTED


def test_rocblas_rules_without_device_work():
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    with hb.RocHandle() as h:
        # m <= 0 (src/vkblas_hipblas.c:838)
        assert vk.lib.rocblas_gemm_ex(h.h, 111, 111, 0, 4, 4, al, 0, 150, 4, 0, 150, 4, be, 0,
                                      150, 4, 0, 150, 4, 151, 0, 0, 0) == vk.rocblas_status_invalid_value
        # c != d -> forwarded -> not_implemented (src/vkblas_hipblas.c:840-843)
        assert vk.lib.rocblas_gemm_ex(h.h, 111, 111, 4, 4, 4, al, 0, 150, 4, 0, 150, 4, be, 16,
                                      150, 4, 32, 150, 4, 151, 0, 0, 0) == \
            vk.rocblas_status_not_implemented
        # compute type must be f32_r
        assert vk.lib.rocblas_gemm_ex(h.h, 111, 111, 4, 4, 4, al, 0, 150, 4, 0, 150, 4, be, 16,
                                      150, 4, 16, 150, 4, 150, 0, 0, 0) == \
            vk.rocblas_status_not_implemented


def _roc_sb(h, m=4, n=4, k=4, c=16, d=16, ldc=4, ldd=4, sc=16, sd=16, batch=2, dt=150, comp=151):
    """rocblas_gemm_strided_batched_ex with dummy pointers (nothing is dereferenced
    on a path that validates or forwards)."""
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    return vk.lib.rocblas_gemm_strided_batched_ex(
        h.h, 111, 111, m, n, k, al, 0x1000, dt, 4, 16, 0x2000, dt, 4, 16, be, c, dt, ldc, sc, d, dt,
        ldd, sd, batch, comp, 0, 0, 0)


def test_rocblas_strided_batched_rules_without_device_work():
    """rocblas_gemm_strided_batched_ex (src/vkblas_hipblas.c:893-955): sizes are
    checked first; only in-place calls with fp32 compute reach the engine, and
    everything else is forwarded (not_implemented without a real rocBLAS)."""
    with hb.RocHandle() as h:
        assert _roc_sb(h, m=0) == vk.rocblas_status_invalid_value        # :902
        assert _roc_sb(h, k=-1) == vk.rocblas_status_invalid_value
        assert _roc_sb(h, batch=0) == vk.rocblas_status_invalid_value
        nimpl = vk.rocblas_status_not_implemented
        assert _roc_sb(h, d=32) == nimpl                                   # c != d
        assert _roc_sb(h, ldd=8) == nimpl                                  # ldc != ldd
        assert _roc_sb(h, comp=150) == nimpl                               # compute f16
        assert _roc_sb(h, dt=170) == nimpl                                 # unknown dtype
        assert _roc_sb(h, sd=32) == nimpl                                  # strideC != strideD
    assert vk.lib.rocblas_gemm_strided_batched_ex(
        None, 111, 111, 4, 4, 4, None, 0, 150, 4, 16, 0, 150, 4, 16, None, 16, 150, 4, 16, 16, 150,
        4, 16, 2, 151, 0, 0, 0) == vk.rocblas_status_invalid_value        # no handle


def test_engine_validation_and_no_device():
    p = 0x10000
    assert vk.gemm(vk.DT_F32, 0, 0, 0, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4) == vk.VKBLAS_ERR_PARAM
    assert vk.gemm(vk.DT_F16, 0, 0, 4, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4, 2, -1, 0, 0) == vk.VKBLAS_ERR_PARAM
    assert vk.gemm(vk.DT_F32, 0, 0, 4, 4, 4, 1.0, 0, 4, p, 4, 0.0, p, 4) == vk.VKBLAS_ERR_PARAM
    assert vk.lib.vkblas_gemm_c64(0, 0, 4, 4, 4, C.c_float(1), C.c_float(0), None, 4, None, 4,
                                  C.c_float(0), C.c_float(0), None, 4, 1, 0, 0, 0) != 0
    vk.lib.vkblas_cache_invalidate_base(None)


def test_replicated_gemm_argument_checks_without_device_work():
    """vkblas_b200_gemm_replicated rejects bad peer lists and problems before
    it looks for a device (these pointers are never dereferenced)."""
    p = 0x10000
    n0 = vk.launch_count()
    ok = dict(A=p, lda=64, B=p, ldb=64, C_=p, ldc=64)

    def call(dtype=vk.DT_F16, M=64, N=64, K=64, peers=(p + 0x1000,), **kw):
        a = {**ok, **kw}
        return vk.gemm_replicated(dtype, 0, 0, M, N, K, 1.0, a["A"], a["lda"], a["B"], a["ldb"],
                                  0.0, a["C_"], a["ldc"], list(peers))
    assert call(peers=[p + 0x1000 * i for i in range(1, 9)]) == vk.VKBLAS_ERR_PARAM   # 8 peers
    assert call(peers=(p, 0)) == vk.VKBLAS_ERR_PARAM                                  # a null peer
    assert call(dtype=7) == vk.VKBLAS_ERR_PARAM                                       # dtype
    assert call(M=0) == vk.VKBLAS_ERR_PARAM
    assert call(C_=0) == vk.VKBLAS_ERR_PARAM
    # a null peer array with a non-zero count
    assert vk.lib.vkblas_b200_gemm_replicated(vk.DT_F16, 0, 0, 64, 64, 64, 1.0, p, 64, p, 64, 0.0,
                                              p, 64, 1, 0, 0, 0, None, 1, None) == vk.VKBLAS_ERR_PARAM
    assert vk.launch_count() == n0


def test_engine_without_gpu_fails_loudly():
    """On a machine with no CUDA device the engine reports ERR_INIT and runs nothing."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    n0 = vk.launch_count()
    st = vk.gemm(vk.DT_F32, 0, 0, 4, 4, 4, 1.0, 0x10000, 4, 0x10000, 4, 0.0, 0x10000, 4)
    assert st == vk.VKBLAS_ERR_INIT
    assert vk.launch_count() == n0


def test_shard_range_covers_exactly_once():
    for units in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 4, 8):
            for block in (1, 64, 128):
                seen = []
                for r in range(world):
                    b, n = vk.shard_range(units, r, world, block)
                    seen.extend(range(b, b + n))
                    if n and block > 1 and b + n < units:
                        assert n % block == 0
                assert seen == list(range(units))
    with pytest.raises(vk.VkblasError):
        vk.shard_range(10, 2, 2)


def test_forwarding_uses_the_real_handle(tmp_path):
    """With a real library present, unhandled calls reach it with ITS handle."""
    so = tmp_path / "libfakehipblas.so"
    src = os.path.join(ROOT, "tests", "fake_real", "fake_hipblas.c")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so), src], check=True)
    code = textwrap.dedent(f"""
        import ctypes as C, sys
        sys.path.insert(0, {ROOT!r})
        import vkblas_b200 as vk
        from vkblas_b200 import hipblas as hb
        fake = C.CDLL({str(so)!r})
        with hb.Handle() as h:
            r = C.c_float(0)
            assert vk.lib.hipblasSdot(h.h, 4, 0, 1, 0, 1, C.byref(r)) == 0, "sdot"
            assert r.value == 42.0 and fake.fake_get_last_call() == 1
            v = C.c_int()
            assert vk.lib.hipblasGetVersion(h.h, C.byref(v)) == 0 and v.value == 424242
            al = (C.c_double * 1)(1.0)
            assert vk.lib.hipblasDgemm(h.h, 111, 111, 4, 4, 4, al, 0, 4, 0, 4, al, 0, 4) == 0
            assert fake.fake_get_last_call() == 3
            assert vk.lib.hipblasStatusToString(0) == b"fake-status"
        with hb.RocHandle() as h:
            a1, b0 = hb.fptr(1.0), hb.fptr(0.0)
            st = vk.lib.rocblas_gemm_ex(h.h, 111, 111, 4, 4, 4, a1, 0, 150, 4, 0, 150, 4, b0, 16,
                                        150, 4, 32, 150, 4, 151, 0, 0, 0)
            assert st == 0 and fake.fake_get_last_call() == 5
            # strided-batched: strideC != strideD is not in place -> forwarded with
            # the caller's strides; an in-place call the engine cannot run (no
            # GPU here) is forwarded too (src/vkblas_hipblas.c:951-954)
            fake.fake_get_last_stride.restype = C.c_longlong
            for sd, want in ((32, 32), (16, 16)):
                st = vk.lib.rocblas_gemm_strided_batched_ex(
                    h.h, 111, 111, 4, 4, 4, a1, 0x1000, 150, 4, 16, 0x2000, 150, 4, 16, b0, 0x3000,
                    150, 4, 16, 0x3000, 150, 4, sd, 2, 151, 0, 0, 0)
                assert st == 0 and fake.fake_get_last_call() == 6, (sd, st)
                assert fake.fake_get_last_stride(3) == want
        print("OK")
    """)
    env = dict(os.environ, VKBLAS_REAL_HIPBLAS=str(so), VKBLAS_REAL_ROCBLAS=str(so))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
