"""Build libvkblas_hipblas.so in-tree (nvcc, sm_100a).

    python -m vkblas_b200.build            # incremental
    python -m vkblas_b200.build --clean    # from scratch

Every .cu is compiled with ``-gencode arch=compute_100a,code=sm_100a`` (the
only target: tcgen05 and TMA need the arch-specific variant), the shim .cpp
with the host compiler, and the objects are linked into one shared library
that statically contains the CUDA runtime and exports only the vkblas_*,
hipblas* and rocblas_* entry points (a version script hides the rest, so
an LD_PRELOAD of this library never interposes the application's own CUDA
runtime).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libvkblas_hipblas.so")
# cuBLAS GEMM interposer for LD_PRELOAD into CUDA applications: the same engine
# objects plus cublas_shim.cpp, exporting only cublas* (under the real
# library's version name, which is what applications bind) and its counter.
CUBLAS_LIB = os.path.join(PKG, "libvkblas_cublas.so")
CUBLAS_SHIM = "cublas_shim"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
            "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-I" + INCLUDE,
             "-I/usr/local/cuda/include"]

VERSION_SCRIPT = """{
  global:
    vkblas_*;
    hipblas*;
    rocblas_*;
  local:
    *;
};
"""

CUBLAS_VERSION_SCRIPT = """libcublas.so.12 {
  global:
    cublas*;
};
VKBLAS_CUBLAS_1 {
  global:
    vkblas_cublas_calls;
  local:
    *;
};
"""


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(f for f in os.listdir(CSRC) if f.endswith(".cpp"))
    hdr = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdr += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return cu, cpp, hdr


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cu, cpp, hdr = _sources()
    jobs = []
    objs = []
    for f in cu:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-3] + ".o")
        objs.append(obj)
        if _stale(obj, [src, __file__] + hdr) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([NVCC, *ARCH, *CU_FLAGS, *extra, "-c", src, "-o", obj])
    for f in cpp:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-4] + ".o")
        objs.append(obj)
        if _stale(obj, [src, __file__] + hdr):
            jobs.append(["g++", *CXX_FLAGS, "-c", src, "-o", obj])
    log = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for out in ex.map(_run, jobs):
            if out.strip():
                log.append(out)
    shim = os.path.join(BUILD, CUBLAS_SHIM + ".o")
    hip_objs = [o for o in objs if o != shim]
    cub_objs = [o for o in objs if not o.endswith("hipblas_shim.o")]
    for lib, lib_objs, script, name in ((LIB, hip_objs, VERSION_SCRIPT, "exports.map"),
                                        (CUBLAS_LIB, cub_objs, CUBLAS_VERSION_SCRIPT,
                                         "exports_cublas.map")):
        if not (jobs or not os.path.exists(lib) or _stale(lib, lib_objs)):
            continue
        vs = os.path.join(BUILD, name)
        with open(vs, "w") as fh:
            fh.write(script)
        tmp = lib + ".tmp"
        # -Bsymbolic-functions: the library's own calls (the shims into the
        # engine) bind inside it, whatever else the process has loaded.
        _run([NVCC, *ARCH, "-shared", "-o", tmp, *lib_objs, "-cudart", "static",
              "-Xlinker", "--version-script=" + vs, "-Xlinker", "-Bsymbolic-functions",
              "-ldl", "-lpthread", "-lrt"])
        os.replace(tmp, lib)
    text = "\n".join(log)
    if verbose and text:
        print(text)
    return text


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args(argv)
    if a.clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    out = build(verbose=True, ptxas_info=a.ptxas_info)
    print("built", LIB)
    return 0 if out is not None else 1


if __name__ == "__main__":
    sys.exit(main())
