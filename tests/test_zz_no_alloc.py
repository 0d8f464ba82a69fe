"""The split-K GEMV entry point that allocates nothing (vkblas_gemv_splitk_noalloc).

It exists for callers that must not have a library call cudaMalloc -- code
running inside a framework's allocator or memory pool, and decode loops that
cannot afford the device-wide synchronisation of a workspace being freed and
reallocated.  Its scratch is a fixed array inside the library, shared by all
calls on a device.  This file is collected last, so a run that stops at the
first failure has run every other test before it.

Checked through the C ABI on a B200, over three calls in a row (the third
needs more per-row-block tickets than the two before it, so it relies on the
per-call ticket clear):

* bit for bit equal to the regular entry point (vkblas_gemm_f16 / _bf16 on
  the GEMV path with the same split-K factor): both run the same kernel with
  the same segments, so any difference would be a mix-up of partial sums or
  tickets in the shared array;
* within the GEMV tolerance of the double-precision oracle (relative
  Frobenius error <= 2e-3 fp16, 8e-3 bf16) and within 0.02 of the
  reference's split-K segment model (segment partials added in order,
  splitk_reduce_half.comp:16-35).  The segment model is not a bit-exact bar:
  inside a segment the kernel's mma.sync instructions add products in their
  own order;
* free device memory is the same before and after the calls;
* sizes beyond the fixed scratch are rejected before anything runs.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev_u16, host_u16  # noqa: E402

CASES = [  # dtype, M, N, K, splitk, alpha, beta
    (vk.DT_F16, 4, 14336, 4096, 4, 1.0, 0.0),        # 896 row blocks
    (vk.DT_BF16, 16, 4096, 4096, 8, 0.5, -1.0),      # 256 row blocks
    (vk.DT_F16, 1, 32768, 2048, 16, 1.5, 0.25),      # 2048 row blocks: more tickets than before
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
        assert vk.last_path() == vk.PATH_GEMV and vk.last_split() == splitk
    finally:
        vk.set_splitk(0)
        vk.set_path(vk.PATH_AUTO)
    assert st == vk.VKBLAS_OK
    return host_u16(dC)


def test_noalloc_gemv_calls_in_a_row(cuda):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    inputs = []
    for i, (dtype, M, N, K, splitk, alpha, beta) in enumerate(CASES):
        dt = 1 if dtype == vk.DT_BF16 else 0
        X, W, C0 = _inputs(dt, M, N, K, 100 + i)
        inputs.append((X, W, C0, dev_u16(X, dt), dev_u16(W, dt), dev_u16(C0, dt)))
    # One untimed call first: it looks up the array's address and loads the
    # library's kernels, so memory is compared over the calls after it.
    dtype, M, N, K, splitk, alpha, beta = CASES[0]
    warm = dev_u16(inputs[0][2], 0)
    assert vk.lib.vkblas_gemv_splitk_noalloc(dtype, M, N, K, alpha, inputs[0][3].data_ptr(), K,
                                             inputs[0][4].data_ptr(), K, beta, warm.data_ptr(), N,
                                             splitk, stream) == vk.VKBLAS_OK
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for i, (dtype, M, N, K, splitk, alpha, beta) in enumerate(CASES):
        dX, dW, dC = inputs[i][3:]
        st = vk.lib.vkblas_gemv_splitk_noalloc(dtype, M, N, K, alpha, dX.data_ptr(), K,
                                               dW.data_ptr(), K, beta, dC.data_ptr(), N, splitk,
                                               stream)
        assert st == vk.VKBLAS_OK, f"call {i}: status {st}"
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "device memory changed across the calls"
    for i, (dtype, M, N, K, splitk, alpha, beta) in enumerate(CASES):
        dt = 1 if dtype == vk.DT_BF16 else 0
        X, W, C0, dX, dW, dC = inputs[i]
        got_bits = host_u16(dC)
        want_bits = _regular(dtype, M, N, K, splitk, alpha, beta, dX, dW, C0, dt)
        assert np.array_equal(got_bits, want_bits), f"call {i}: differs from the regular entry point"
        got = orc.widen(dt, got_bits).reshape(M, N)
        ref = orc.hgemm_rowmajor_f64(dt, 0, 1, M, N, K, alpha, X, K, W, K, beta, C0, N)[0]
        err = orc.rel_frobenius(got, ref)
        assert err <= (8e-3 if dt else 2e-3), f"call {i}: relative error {err}"
        seg = C0.copy()
        orc.hgemm_rowmajor_splitk(dt, 0, 1, M, N, K, splitk, alpha, X, K, W, K, beta, seg, N)
        assert np.max(np.abs(got - orc.widen(dt, seg).reshape(M, N))) <= 0.02, f"call {i}"


def test_noalloc_gemv_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    M, N, K = 16, 14336, 4096          # 8 x 16 x 14336 x 4 bytes of partials > 4 MiB
    dX = torch.zeros(M * K, device="cuda", dtype=torch.float16)
    dW = torch.zeros(N * K, device="cuda", dtype=torch.float16)
    dC = torch.full((M * N,), 3.0, device="cuda", dtype=torch.float16)
    st = vk.lib.vkblas_gemv_splitk_noalloc(vk.DT_F16, M, N, K, 1.0, dX.data_ptr(), K,
                                           dW.data_ptr(), K, 0.0, dC.data_ptr(), N, 8, stream)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_ERR_PARAM
    # more row blocks (16 weight rows each) than the array has tickets
    n_big = 16384 * 16 + 16
    dWb = torch.zeros(n_big * 64, device="cuda", dtype=torch.float16)
    dCb = torch.full((n_big,), 3.0, device="cuda", dtype=torch.float16)
    st = vk.lib.vkblas_gemv_splitk_noalloc(vk.DT_F16, 1, n_big, 64, 1.0, dX.data_ptr(), 64,
                                           dWb.data_ptr(), 64, 0.0, dCb.data_ptr(), n_big, 2,
                                           stream)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_ERR_PARAM
    assert bool((dC == 3.0).all()) and bool((dCb == 3.0).all()), "a rejected call must not touch C"
