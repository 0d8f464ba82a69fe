"""cuBLAS interposer (libvkblas_cublas.so) without a GPU.

* it exports exactly the intercepted GEMM entry points, under the real
  library's symbol version (libcublas.so.12, what applications bind), plus its
  call counter -- no engine or CUDA runtime names;
* with no usable GPU every GEMM is declined and reaches the real library
  (here a recording fake) with the caller's handle and arguments unchanged;
* empty and invalid problems go to the real library without touching the
  engine.
The interception itself (PyTorch `a @ b` under LD_PRELOAD running on this
library's kernels) is tested on the GPU in test_cublas_preload_gpu.py.
"""
import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "vkblas_b200", "libvkblas_cublas.so")

INTERCEPTED = ["cublasSgemm_v2", "cublasSgemmStridedBatched", "cublasSgemmEx", "cublasGemmEx",
               "cublasGemmStridedBatchedEx", "cublasHgemm", "cublasHgemmStridedBatched"]


def _dynsyms():
    out = subprocess.run(["nm", "-D", "--defined-only", "--with-symbol-versions", SHIM],
                         capture_output=True, text=True, check=True).stdout
    syms = {}
    for line in out.splitlines():
        parts = line.split()
        if len(parts) == 3 and parts[1] in "TtWw":
            name, _, ver = parts[2].partition("@@")
            syms[name] = ver
    return syms


def test_exports_are_the_intercepted_entry_points_only():
    syms = _dynsyms()
    assert set(syms) == set(INTERCEPTED) | {"vkblas_cublas_calls"}, sorted(syms)
    for name in INTERCEPTED:
        assert syms[name] == "libcublas.so.12", (name, syms[name])


def test_header_declarations_are_exported():
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_abi import _declared_functions
    decl = _declared_functions(headers={"vkblas_cublas.h"})
    assert decl == ["vkblas_cublas_calls"]
    assert set(decl) <= set(_dynsyms())


@pytest.fixture(scope="module")
def fake_cublas(tmp_path_factory):
    so = tmp_path_factory.mktemp("fake") / "libfake_cublas.so"
    src = os.path.join(ROOT, "tests", "fake_real", "fake_cublas.c")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so), src], check=True)
    return str(so)


SCRIPT = textwrap.dedent(r"""
    import ctypes as C, json, sys
    fake = C.CDLL(sys.argv[1])
    shim = C.CDLL(sys.argv[2])
    H = C.c_void_p(0xC0B1)
    f1, f0 = C.c_float(1.0), C.c_float(0.0)
    buf = (C.c_float * 64)()
    p = C.cast(buf, C.c_void_p)
    ll = C.c_longlong
    res = {}
    def last():
        return [C.c_int.in_dll(fake, "fake_last").value] + list((C.c_longlong * 12).in_dll(fake, "fake_args"))[:10]
    st = shim.cublasSgemm_v2(H, 0, 1, 4, 5, 6, C.byref(f1), p, 4, p, 5, C.byref(f0), p, 4)
    res["sgemm"] = [st] + last()
    st = shim.cublasSgemmStridedBatched(H, 0, 0, 4, 5, 6, C.byref(f1), p, 4, ll(24), p, 6, ll(30),
                                        C.byref(f0), p, 4, ll(20), 3)
    res["sgemm_sb"] = [st] + last()
    st = shim.cublasSgemmEx(H, 1, 0, 4, 5, 6, C.byref(f1), p, 2, 6, p, 2, 6, C.byref(f0), p, 0, 4)
    res["sgemmex_mixed"] = [st] + last()
    st = shim.cublasGemmEx(H, 0, 0, 4, 5, 6, C.byref(f1), p, 2, 4, p, 2, 6, C.byref(f0), p, 2, 4,
                           68, -1)
    res["gemmex"] = [st] + last()
    st = shim.cublasGemmEx(H, 0, 0, 4, 5, 6, C.byref(f1), p, 2, 4, p, 2, 6, C.byref(f0), p, 2, 4,
                           64, 99)
    res["gemmex_16f"] = [st] + last()
    st = shim.cublasGemmStridedBatchedEx(H, 0, 0, 4, 5, 6, C.byref(f1), p, 14, 4, ll(24), p, 14, 6,
                                         ll(30), C.byref(f0), p, 14, 4, ll(20), 2, 68, -1)
    res["gemm_sb_ex"] = [st] + last()
    h1 = (C.c_uint16 * 1)(0x3C00)
    st = shim.cublasHgemm(H, 0, 0, 4, 5, 6, h1, p, 4, p, 6, h1, p, 4)
    res["hgemm"] = [st] + last()
    st = shim.cublasHgemmStridedBatched(H, 0, 0, 4, 5, 6, h1, p, 4, ll(24), p, 6, ll(30), h1, p, 4,
                                        ll(20), 2)
    res["hgemm_sb"] = [st] + last()
    st = shim.cublasSgemm_v2(H, 0, 0, 4, 5, 0, C.byref(f1), p, 4, p, 1, C.byref(f0), p, 4)
    res["k0"] = [st] + last()
    st = shim.cublasSgemm_v2(H, 0, 0, 4, 5, 6, C.byref(f1), p, 3, p, 6, C.byref(f0), p, 4)
    res["bad_lda"] = [st] + last()
    shim.vkblas_cublas_calls.restype = C.c_ulonglong
    res["ran"] = shim.vkblas_cublas_calls(0)
    res["forwarded"] = shim.vkblas_cublas_calls(1)
    print(json.dumps(res))
""")


def test_declined_calls_reach_the_real_library_unchanged(fake_cublas, tmp_path):
    import json
    script = tmp_path / "fwd.py"
    script.write_text(SCRIPT)
    env = dict(os.environ, VKBLAS_REAL_CUBLAS=fake_cublas, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(script), fake_cublas, SHIM], env=env,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    r = json.loads(out.stdout.strip().splitlines()[-1])
    # [status, which, m, n, k, lda, ldb, ldc, type/batch, compute, algo, strideC]
    assert r["sgemm"][:8] == [0, 1, 4, 5, 6, 4, 5, 4]
    assert r["sgemm_sb"][:9] == [0, 2, 4, 5, 6, 4, 6, 4, 3] and r["sgemm_sb"][11] == 20
    assert r["sgemmex_mixed"][:2] == [0, 3] and r["sgemmex_mixed"][8] == 2 * 100 + 0
    assert r["gemmex"][:2] == [0, 4] and r["gemmex"][8:11] == [202, 68, -1]
    assert r["gemmex_16f"][:2] == [0, 4] and r["gemmex_16f"][9:11] == [64, 99]
    assert r["gemm_sb_ex"][:2] == [0, 5] and r["gemm_sb_ex"][8:12] == [2, 68, -1, 20]
    assert r["hgemm"][:2] == [0, 6]
    assert r["hgemm_sb"][:2] == [0, 7] and r["hgemm_sb"][8] == 2
    assert r["k0"][:5] == [0, 1, 4, 5, 0]
    assert r["bad_lda"][:2] == [0, 1] and r["bad_lda"][5] == 3
    assert r["ran"] == 0 and r["forwarded"] == 10
