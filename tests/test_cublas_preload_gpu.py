"""cuBLAS interposer on the GPU: PyTorch matmuls under LD_PRELOAD run on this
library's kernels and agree with double.

A fresh interpreter is started with LD_PRELOAD=libvkblas_cublas.so (the only
way to interpose cuBLAS under PyTorch, whose libraries bind the versioned
libcublas.so.12 symbols).  It runs fp32 / fp16 / bf16 matmuls, transposed
views and batched matmuls through torch's cuBLAS backend, and reads the
interposer's counters: every one of those calls must have run here.  An fp64
matmul (not intercepted) must still be right.
"""
import json
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "vkblas_b200", "libvkblas_cublas.so")

SCRIPT = textwrap.dedent(r"""
    import ctypes, json, sys
    import torch
    shim = ctypes.CDLL(sys.argv[1])          # already preloaded: the same instance
    shim.vkblas_cublas_calls.restype = ctypes.c_uint64
    torch.backends.cuda.preferred_blas_library("cublas")
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(0)
    out = {}

    def check(name, fn, *xs):
        n0 = shim.vkblas_cublas_calls(0)
        y = fn(*xs)
        torch.cuda.synchronize()
        ran = shim.vkblas_cublas_calls(0) - n0
        ref = fn(*[x.double().cpu() for x in xs])
        err = ((y.double().cpu() - ref).norm() / ref.norm()).item()
        out[name] = [int(ran), err]

    for dt in (torch.float32, torch.float16, torch.bfloat16):
        a = torch.randn(512, 384, device="cuda", dtype=dt, generator=g)
        b = torch.randn(384, 320, device="cuda", dtype=dt, generator=g)
        check(f"mm_{dt}", torch.matmul, a, b)
        check(f"mm_tt_{dt}", lambda x, y: x.t() @ y.t(), b, a)
    for dt in (torch.float32, torch.float16):
        x = torch.randn(6, 256, 192, device="cuda", dtype=dt, generator=g)
        y = torch.randn(6, 192, 130, device="cuda", dtype=dt, generator=g)
        check(f"bmm_{dt}", torch.bmm, x, y)
    a = torch.randn(64, 48, device="cuda", dtype=torch.float64, generator=g)
    b = torch.randn(48, 40, device="cuda", dtype=torch.float64, generator=g)
    check("mm_f64", torch.matmul, a, b)
    out["forwarded"] = int(shim.vkblas_cublas_calls(1))
    print(json.dumps(out))
""")

TOL = {"torch.float32": 1e-5, "torch.float16": 2e-3, "torch.bfloat16": 8e-3}


def test_torch_matmul_runs_on_the_interposer(tmp_path):
    script = tmp_path / "preload.py"
    script.write_text(SCRIPT)
    env = dict(os.environ, LD_PRELOAD=SHIM)
    p = subprocess.run([sys.executable, str(script), SHIM], env=env, capture_output=True,
                       text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    for name, val in r.items():
        if name in ("forwarded", "mm_f64"):
            continue
        ran, err = val
        dt = name.rsplit("_", 1)[-1]
        assert ran >= 1, f"{name}: not run by the interposer ({r})"
        assert err <= TOL[dt], f"{name}: relative error {err}"
    assert r["mm_f64"][0] == 0 and r["mm_f64"][1] <= 1e-12
