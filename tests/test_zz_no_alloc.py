"""The split-K GEMV entry point that allocates nothing (vkblas_gemv_splitk_noalloc).

It exists for callers that must not have a library call cudaMalloc -- code
running inside a framework's allocator or memory pool, and decode loops that
cannot afford the device-wide synchronisation of a workspace being freed and
reallocated.  Its scratch is a fixed array inside the library, shared by all
calls on a device.  This file is collected last, so a run that stops at the
first failure has run every other test before it.

Checked through the C ABI on a B200: two calls in a row, each compared with
the regular entry point (vkblas_gemm_f16 / _bf16, same split-K) within the
GEMV tolerance (relative Frobenius error <= 2e-3 fp16, 8e-3 bf16), and the
size limit rejected before anything runs.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev_u16, host_u16  # noqa: E402

CASES = [  # dtype, M, N, K, splitk, alpha, beta
    (vk.DT_F16, 4, 14336, 4096, 4, 1.0, 0.0),
    (vk.DT_BF16, 16, 4096, 4096, 8, 0.5, -1.0),
]


def _inputs(dt, M, N, K, seed):
    rng = np.random.default_rng(seed)
    X = orc.narrow(dt, rng.uniform(-1, 1, M * K).astype(np.float32))
    W = orc.narrow(dt, (rng.standard_normal(N * K) * 0.05).astype(np.float32))
    C0 = orc.narrow(dt, rng.uniform(-1, 1, M * N).astype(np.float32))
    return X, W, C0


def _regular(dtype, M, N, K, splitk, alpha, beta, dX, dW, C0, dt):
    import torch
    dC = dev_u16(C0, dt)
    vk.set_path(vk.PATH_GEMV)
    vk.set_splitk(splitk)
    try:
        vk.set_stream(torch.cuda.current_stream())
        st = vk.gemm(dtype, vk.OP_N, vk.OP_T, M, N, K, alpha, dX.data_ptr(), K, dW.data_ptr(), K,
                     beta, dC.data_ptr(), N)
        torch.cuda.synchronize()
    finally:
        vk.set_splitk(0)
        vk.set_path(vk.PATH_AUTO)
    assert st == vk.VKBLAS_OK
    return orc.widen(dt, host_u16(dC)).reshape(M, N)


def test_noalloc_gemv_two_calls_match_regular_entry_point(cuda):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    for i, (dtype, M, N, K, splitk, alpha, beta) in enumerate(CASES):   # two calls in a row
        dt = 1 if dtype == vk.DT_BF16 else 0
        X, W, C0 = _inputs(dt, M, N, K, 100 + i)
        dX, dW, dC = dev_u16(X, dt), dev_u16(W, dt), dev_u16(C0, dt)
        st = vk.lib.vkblas_gemv_splitk_noalloc(dtype, M, N, K, alpha, dX.data_ptr(), K,
                                               dW.data_ptr(), K, beta, dC.data_ptr(), N, splitk,
                                               stream)
        torch.cuda.synchronize()
        assert st == vk.VKBLAS_OK, f"call {i}: status {st}"
        got = orc.widen(dt, host_u16(dC)).reshape(M, N)
        want = _regular(dtype, M, N, K, splitk, alpha, beta, dX, dW, C0, dt)
        err = orc.rel_frobenius(got, want)
        assert err <= (8e-3 if dt else 2e-3), f"call {i}: relative error {err}"


def test_noalloc_gemv_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    M, N, K = 16, 14336, 4096          # 8 x 16 x 14336 x 4 bytes of partials > 4 MiB
    dX = torch.zeros(M * K, device="cuda", dtype=torch.float16)
    dW = torch.zeros(N * K, device="cuda", dtype=torch.float16)
    dC = torch.full((M * N,), 3.0, device="cuda", dtype=torch.float16)
    st = vk.lib.vkblas_gemv_splitk_noalloc(vk.DT_F16, M, N, K, 1.0, dX.data_ptr(), K,
                                           dW.data_ptr(), K, 0.0, dC.data_ptr(), N, 8,
                                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_ERR_PARAM
    assert bool((dC == 3.0).all()), "a rejected call must not touch C"
