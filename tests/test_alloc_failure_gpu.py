"""Scratch-memory failure, injected on the host (vkblas_b200_set_test_alloc_fail).

The reference engine grows its workspace on demand and, when a call cannot
run, returns an error so that its hipBLAS shim forwards the call to the real
library (src/vkblas.c:1888-1914, src/vkblas_hipblas.c:244-246).  Here a scratch
request that fails as a failed cudaMalloc would must never give a wrong
result and never touch the GPU in a faulting way:

* automatic path: an fp32 GEMM that cannot get its 3xTF32 operand planes runs
  on the exact SIMT kernel (bit-exact against the sequential oracle); a
  tensor-core HGEMM or a GEMV that cannot get split-K scratch runs unsplit;
* path forced to the tensor cores: VKBLAS_ERR_FALLBACK, C untouched; through
  hipblasSgemm the shim then forwards, i.e. HIPBLAS_STATUS_NOT_SUPPORTED
  without a real hipBLAS, C untouched;
* complex64: non-zero status (the caller falls back), C untouched;
* after the hook is cleared the same calls run normally.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import hipblas as hb  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev, host, dev_u16, host_u16, check_status  # noqa: E402


@pytest.fixture
def alloc_fail():
    vk.lib.vkblas_b200_set_test_alloc_fail(-1)
    try:
        yield
    finally:
        vk.lib.vkblas_b200_set_test_alloc_fail(0)
        vk.set_path(vk.PATH_AUTO)
        vk.set_splitk(0)


def _sgemm_inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    C0 = rng.uniform(-1, 1, M * N).astype(np.float32)
    return A, B, C0


def test_fp32_without_planes_runs_exact_kernel(cuda, alloc_fail):
    import torch
    M, N, K = 512, 384, 256
    A, B, C0 = _sgemm_inputs(M, N, K, 1)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    vk.set_stream(torch.cuda.current_stream())
    st = vk.gemm(vk.DT_F32, 0, 0, M, N, K, 1.5, dA.data_ptr(), K, dB.data_ptr(), N, 0.5,
                 dC.data_ptr(), N)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_SIMT
    want = C0.copy()
    orc.gemm_rowmajor_f32seq(0, 0, M, N, K, 1.5, A, K, B, N, 0.5, want, N)
    assert np.array_equal(host(dC).view(np.uint32), want.view(np.uint32))
    check_status()


def test_forced_tensor_core_path_declines_and_shim_forwards(cuda, alloc_fail):
    import torch
    M, N, K = 512, 384, 256
    A, B, C0 = _sgemm_inputs(M, N, K, 2)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    vk.set_path(vk.PATH_TC)
    vk.set_stream(torch.cuda.current_stream())
    st = vk.gemm(vk.DT_F32, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0,
                 dC.data_ptr(), N)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_ERR_FALLBACK
    # hipBLAS column-major view of the same call: forwarded, nothing to forward to
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    with hb.Handle() as h:
        h.set_stream(torch.cuda.current_stream())
        hs = vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, N, M, K, al,
                                 dB.data_ptr(), N, dA.data_ptr(), K, be, dC.data_ptr(), N)
        torch.cuda.synchronize()
    assert hs == vk.HIPBLAS_STATUS_NOT_SUPPORTED
    assert np.array_equal(host(dC), C0), "a declined call must not touch C"
    vk.lib.vkblas_b200_set_test_alloc_fail(0)
    st = vk.gemm(vk.DT_F32, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0,
                 dC.data_ptr(), N)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_TC
    want = orc.gemm_rowmajor_f64(0, 0, M, N, K, 1.0, A, K, B, N, 0.0, None, N)[0]
    assert orc.rel_frobenius(host(dC).reshape(M, N), want) <= 1e-5


def test_split_k_without_scratch_runs_unsplit(cuda, alloc_fail):
    import torch
    vk.set_stream(torch.cuda.current_stream())
    rng = np.random.default_rng(3)
    # tensor-core HGEMM that would split its K range 16 ways (256 x 256 x 4096)
    M, N, K = 256, 256, 4096
    A = orc.f2h(rng.uniform(-1, 1, M * K).astype(np.float32))
    B = orc.f2h(rng.uniform(-1, 1, N * K).astype(np.float32))
    dA, dB, dC = dev_u16(A, 0), dev_u16(B, 0), dev_u16(np.zeros(M * N, np.uint16), 0)
    st = vk.gemm(vk.DT_F16, 0, 1, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), K, 0.0,
                 dC.data_ptr(), N)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_TC and vk.last_split() == 1
    want = orc.hgemm_rowmajor_f64(0, 0, 1, M, N, K, 1.0, A, K, B, K, 0.0, None, N)[0]
    assert orc.rel_frobenius(orc.h2f(host_u16(dC)).reshape(M, N), want) <= 2e-3
    # decode GEMV asked to split 8 ways
    M, N, K = 4, 1024, 4096
    X = orc.f2h(rng.uniform(-1, 1, M * K).astype(np.float32))
    W = orc.f2h(rng.uniform(-1, 1, N * K).astype(np.float32))
    dX, dW, dC = dev_u16(X, 0), dev_u16(W, 0), dev_u16(np.zeros(M * N, np.uint16), 0)
    vk.set_splitk(8)
    st = vk.gemm(vk.DT_F16, 0, 1, M, N, K, 1.0, dX.data_ptr(), K, dW.data_ptr(), K, 0.0,
                 dC.data_ptr(), N)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_GEMV and vk.last_split() == 1
    want = orc.hgemm_rowmajor_f64(0, 0, 1, M, N, K, 1.0, X, K, W, K, 0.0, None, N)[0]
    assert orc.rel_frobenius(orc.h2f(host_u16(dC)).reshape(M, N), want) <= 2e-3
    check_status()


def test_complex_without_planes_reports_failure(cuda, alloc_fail):
    import ctypes as C
    import torch
    M, N, K = 64, 48, 32
    rng = np.random.default_rng(4)
    A = rng.uniform(-1, 1, 2 * M * K).astype(np.float32)
    B = rng.uniform(-1, 1, 2 * K * N).astype(np.float32)
    C0 = rng.uniform(-1, 1, 2 * M * N).astype(np.float32)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    vk.set_stream(torch.cuda.current_stream())
    r = vk.lib.vkblas_gemm_c64(0, 0, M, N, K, C.c_float(1), C.c_float(0), dA.data_ptr(), K,
                               dB.data_ptr(), N, C.c_float(0), C.c_float(0), dC.data_ptr(), N, 1,
                               0, 0, 0)
    torch.cuda.synchronize()
    assert r != 0
    assert np.array_equal(host(dC), C0)
