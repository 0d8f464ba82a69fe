"""fp32 decode GEMV (engine op_a = N, M <= 8, batch 1) against the oracle.

K x N weights (engine op_b = N): bit-identical to the fp32 split-K model
(segments of ceil(K/S) k, each a sequential fmaf sum, added in order) for the
split count S the call reports -- the reference's matvec_f32 TB=0 arithmetic.
N x K weights (engine op_b = T): relative Frobenius error <= 2e-6 against
double, and bit-identical from run to run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev, host, check_status  # noqa: E402


def _call(M, N, K, alpha, X, ldx, W, ldw, beta, C, ldc, op_b, splitk=0):
    import torch
    vk.set_splitk(splitk)
    try:
        vk.set_stream(torch.cuda.current_stream())
        st = vk.gemm(vk.DT_F32, 0, op_b, M, N, K, alpha, X.data_ptr(), ldx, W.data_ptr(), ldw,
                     beta, C.data_ptr(), ldc)
        torch.cuda.synchronize()
    finally:
        vk.set_splitk(0)
    assert st == vk.VKBLAS_OK, st
    check_status()


KN_CASES = [
    (1, 4096, 4096, 0, 0.0),
    (1, 1000, 777, 1, 0.5),
    (3, 1000, 777, 3, 0.5),
    (8, 130, 2048, 8, -1.0),
    (2, 7, 33, 2, 0.5),          # fewer columns than one thread's four
    (1, 14336, 4096, 0, 0.0),    # the decode layer shape, automatic split
]


@pytest.mark.parametrize("case", KN_CASES, ids=[f"{m}x{n}x{k}-s{s}" for m, n, k, s, _ in KN_CASES])
def test_gemv_f32_kn_matches_splitk_model(case, cuda):
    M, N, K, splitk, beta = case
    rng = np.random.default_rng(M * 31 + N + K)
    ldx, ldw, ldc = K + 3, (N + 3) // 4 * 4 + 4, N + 5
    X = rng.uniform(-1, 1, M * ldx).astype(np.float32)
    W = rng.uniform(-1, 1, K * ldw).astype(np.float32)
    C0 = rng.uniform(-1, 1, M * ldc).astype(np.float32)
    dX, dW, dC = dev(X), dev(W), dev(C0)
    _call(M, N, K, 1.5, dX, ldx, dW, ldw, beta, dC, ldc, 0, splitk)
    assert vk.last_path() == vk.PATH_GEMV
    S = vk.last_split()
    if splitk:
        assert S == splitk
    want = C0.copy()
    orc.gemm_rowmajor_f32_splitk(0, 0, M, N, K, -(-K // S), 1.5, X, ldx, W, ldw, beta, want, ldc)
    got = host(dC)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"S={S}: {np.count_nonzero(got != want)} elements differ"


NK_CASES = [(1, 4096, 4096), (5, 1000, 772), (8, 33, 2048), (1, 14336, 4096), (2, 96, 4)]


@pytest.mark.parametrize("shape", NK_CASES, ids=[f"{m}x{n}x{k}" for m, n, k in NK_CASES])
def test_gemv_f32_nk_accuracy_and_determinism(shape, cuda):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N + K)
    ldx, ldw, ldc = K + 4, K + 8, N + 1
    X = rng.uniform(-1, 1, M * ldx).astype(np.float32)
    W = rng.uniform(-1, 1, N * ldw).astype(np.float32)
    C0 = rng.uniform(-1, 1, M * ldc).astype(np.float32)
    outs = []
    for _ in range(2):
        dX, dW, dC = dev(X), dev(W), dev(C0)
        _call(M, N, K, 0.75, dX, ldx, dW, ldw, -0.5, dC, ldc, 1)
        assert vk.last_path() == vk.PATH_GEMV
        outs.append(host(dC))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = orc.gemm_rowmajor_f64(0, 1, M, N, K, 0.75, X, ldx, W, ldw, -0.5, C0, ldc)[0]
    got = outs[0].reshape(M, ldc)
    assert orc.rel_frobenius(got[:, :N], want) <= 2e-6
    np.testing.assert_array_equal(got[:, N:], C0.reshape(M, ldc)[:, N:])


def test_gemv_f32_misaligned_weights_take_another_path(cuda):
    """ldw not a multiple of 4: no 128-bit weight rows, so the call runs on
    another kernel and is still correct."""
    M, N, K = 1, 300, 256
    rng = np.random.default_rng(3)
    ldw = N + 1
    X = rng.uniform(-1, 1, K).astype(np.float32)
    W = rng.uniform(-1, 1, K * ldw).astype(np.float32)
    dX, dW, dC = dev(X), dev(W), dev(np.zeros(N, np.float32))
    _call(M, N, K, 1.0, dX, K, dW, ldw, 0.0, dC, N, 0)
    assert vk.last_path() != vk.PATH_GEMV
    want = orc.gemm_rowmajor_f64(0, 0, M, N, K, 1.0, X, K, W, ldw, 0.0, None, N)[0]
    assert orc.rel_frobenius(host(dC).reshape(M, N), want) <= 1e-5
