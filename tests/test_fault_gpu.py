"""Bounded waits of the tcgen05 GEMM, exercised without faulting the GPU.

The test hook (vkblas_b200_set_test_stall) makes the TMA producer leave the
first shared-memory stage unfilled, a wait nothing will ever satisfy, and
shortens every wait to 20 ms.  The kernel must end by itself: the waiting
role records a timeout code in the device status word, raises the CTA abort
flag, every role unwinds, nothing stays in flight and TMEM is freed.  The same
context must then run a normal GEMM correctly.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev_u16, host_u16  # noqa: E402


def _gemm(dA, dB, dC, M, N, K):
    import torch
    vk.set_stream(torch.cuda.current_stream())
    return vk.gemm(vk.DT_F16, 0, 1, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), K, 0.0,
                   dC.data_ptr(), N)


def test_wait_timeout_is_reported_and_context_survives(cuda):
    import torch
    M, N, K = 256, 512, 256
    rng = np.random.default_rng(0)
    A = orc.f2h(rng.uniform(-1, 1, M * K).astype(np.float32))
    B = orc.f2h(rng.uniform(-1, 1, N * K).astype(np.float32))
    dA, dB = dev_u16(A, 0), dev_u16(B, 0)
    dC = dev_u16(np.zeros(M * N, np.uint16), 0)
    assert vk.device_status(True) == 0
    vk.set_path(vk.PATH_TC)
    try:
        vk.lib.vkblas_b200_set_test_stall(1)
        t0 = time.time()
        assert _gemm(dA, dB, dC, M, N, K) == vk.VKBLAS_OK      # the launch itself is fine
        torch.cuda.synchronize()                              # ... and the kernel ends
        elapsed = time.time() - t0
        vk.lib.vkblas_b200_set_test_stall(0)
        status = vk.device_status(True)
        assert status in (1, 2, 3), f"expected a wait-timeout code, got {status}"
        assert elapsed < 10.0
        # the same context still computes correctly
        assert _gemm(dA, dB, dC, M, N, K) == vk.VKBLAS_OK
        torch.cuda.synchronize()
    finally:
        vk.lib.vkblas_b200_set_test_stall(0)
        vk.set_path(vk.PATH_AUTO)
    assert vk.device_status(True) == 0
    got = orc.h2f(host_u16(dC)).reshape(M, N)
    want = orc.hgemm_rowmajor_f64(0, 0, 1, M, N, K, 1.0, A, K, B, K, 0.0, None, N)[0]
    assert orc.rel_frobenius(got, want) <= 2e-3
