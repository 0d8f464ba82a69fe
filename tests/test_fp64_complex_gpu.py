"""fp64, complex64 and complex128 GEMMs (reference src/vkblas.c:3653-4188 and
the hipBLAS entry points of src/vkblas_hipblas.c:470-620) against the oracle.

fp64 and complex128 are bit-identical to the oracle's restatement of the
reference arithmetic (sequential fma, four real GEMMs on planar copies, the
cx_combine order).  complex64 is bit-identical when its four fp32 GEMMs take
the exact SIMT path, and within 1e-5 (relative Frobenius) on the default
path, whose fp32 GEMMs may run as 3xTF32.  Leading-dimension padding of C
must stay untouched.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import hipblas as hb  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import check_status  # noqa: E402

SHAPES = [(64, 64, 64), (37, 53, 71), (130, 96, 300), (1, 200, 64)]
OPS = [(0, 0), (0, 1), (1, 0), (1, 1)]


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _layout(op_a, op_b, M, N, K, batch=1, bcast=None):
    lda = (M if op_a else K) + 1
    ldb = (K if op_b else N) + 2
    ldc = N + 3
    ra, rb = (K if op_a else M), (N if op_b else K)
    sa = 0 if bcast == "a" else ra * lda
    sb = 0 if bcast == "b" else rb * ldb
    sc = M * ldc
    na = (sa * (batch - 1) if sa else 0) + ra * lda
    nb = (sb * (batch - 1) if sb else 0) + rb * ldb
    nc = sc * (batch - 1) + M * ldc
    return lda, ldb, ldc, sa, sb, sc, na, nb, nc


def _sync_stream():
    import torch
    vk.set_stream(torch.cuda.current_stream())


@pytest.mark.parametrize("ops", OPS, ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_f64_bit_exact(ops, shape, cuda):
    import torch
    M, N, K = shape
    lda, ldb, ldc, sa, sb, sc, na, nb, nc = _layout(*ops, M, N, K)
    rng = np.random.default_rng(M + N + K + ops[0] * 3 + ops[1])
    A, B, C0 = rng.standard_normal(na), rng.standard_normal(nb), rng.standard_normal(nc)
    dA, dB, dC = _dev(A), _dev(B), _dev(C0)
    _sync_stream()
    assert vk.lib.vkblas_gemm_f64(ops[0], ops[1], M, N, K, 1.5, dA.data_ptr(), lda, dB.data_ptr(),
                                  ldb, -0.5, dC.data_ptr(), ldc, 1, 0, 0, 0) == 0
    torch.cuda.synchronize()
    check_status()
    want = C0.copy()
    orc.dgemm_rowmajor_seq(ops[0], ops[1], M, N, K, 1.5, A, lda, B, ldb, -0.5, want, ldc)
    assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))


@pytest.mark.parametrize("bcast", [None, "a", "b"])
def test_f64_batched(bcast, cuda):
    import torch
    M, N, K, batch = 40, 33, 50, 3
    lda, ldb, ldc, sa, sb, sc, na, nb, nc = _layout(0, 1, M, N, K, batch, bcast)
    rng = np.random.default_rng(5)
    A, B, C0 = rng.standard_normal(na), rng.standard_normal(nb), rng.standard_normal(nc)
    dA, dB, dC = _dev(A), _dev(B), _dev(C0)
    _sync_stream()
    assert vk.lib.vkblas_gemm_f64(0, 1, M, N, K, 0.5, dA.data_ptr(), lda, dB.data_ptr(), ldb, 0.0,
                                  dC.data_ptr(), ldc, batch, sa, sb, sc) == 0
    torch.cuda.synchronize()
    want = C0.copy()
    orc.dgemm_rowmajor_seq(0, 1, M, N, K, 0.5, A, lda, B, ldb, 0.0, want, ldc, batch, sa, sb, sc)
    assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))


def test_f64_batch_above_grid_z_limit(cuda):
    """More batch entries than a grid's z extent (65535): the kernel strides over them."""
    import torch
    M, N, K, batch = 3, 2, 5, 70000
    lda, ldb, ldc, sa, sb, sc, na, nb, nc = _layout(0, 0, M, N, K, batch)
    rng = np.random.default_rng(11)
    A, B, C0 = rng.standard_normal(na), rng.standard_normal(nb), rng.standard_normal(nc)
    dA, dB, dC = _dev(A), _dev(B), _dev(C0)
    _sync_stream()
    assert vk.lib.vkblas_gemm_f64(0, 0, M, N, K, 1.25, dA.data_ptr(), lda, dB.data_ptr(), ldb, 0.5,
                                  dC.data_ptr(), ldc, batch, sa, sb, sc) == 0
    torch.cuda.synchronize()
    want = C0.copy()
    orc.dgemm_rowmajor_seq(0, 0, M, N, K, 1.25, A, lda, B, ldb, 0.5, want, ldc, batch, sa, sb, sc)
    assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))


def _cx(rng, n, dt):
    return rng.standard_normal(2 * n).astype(dt)        # interleaved re, im


def _run_cx(dbl, ops, M, N, K, alpha, beta, batch=1, bcast=None, path=None):
    import torch
    dt = np.float64 if dbl else np.float32
    lda, ldb, ldc, sa, sb, sc, na, nb, nc = _layout(*ops, M, N, K, batch, bcast)
    rng = np.random.default_rng(M * 3 + N + K + ops[0] + 2 * ops[1] + batch + int(dbl))
    A, B, C0 = _cx(rng, na, dt), _cx(rng, nb, dt), _cx(rng, nc, dt)
    dA, dB, dC = _dev(A), _dev(B), _dev(C0)
    _sync_stream()
    fn = vk.lib.vkblas_gemm_z64 if dbl else vk.lib.vkblas_gemm_c64
    if path is not None:
        vk.set_path(path)
    try:
        st = fn(ops[0], ops[1], M, N, K, alpha.real, alpha.imag, dA.data_ptr(), lda, dB.data_ptr(),
                ldb, beta.real, beta.imag, dC.data_ptr(), ldc, batch, sa, sb, sc)
        torch.cuda.synchronize()
    finally:
        vk.set_path(vk.PATH_AUTO)
    assert st == 0
    check_status()
    want = C0.copy()
    (orc.zgemm_rowmajor if dbl else orc.cgemm_rowmajor)(ops[0], ops[1], M, N, K, alpha, A, lda, B,
                                                        ldb, beta, want, ldc, batch, sa, sb, sc)
    return dC.cpu().numpy(), want, C0, (ldc, sc, batch, M, N)


@pytest.mark.parametrize("ops", OPS, ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_z64_bit_exact(ops, shape, cuda):
    got, want, _, _ = _run_cx(True, ops, *shape, 0.75 - 1.5j, 0.5 + 0.25j)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))


@pytest.mark.parametrize("ops", OPS, ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_c64_exact_path_bit_exact(ops, shape, cuda):
    got, want, _, _ = _run_cx(False, ops, *shape, 1.25 + 0.5j, -0.75 + 0j, path=vk.PATH_SIMT)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bcast", [None, "a", "b"])
def test_complex_batched_beta_zero(bcast, cuda):
    got, want, _, _ = _run_cx(True, (1, 0), 48, 40, 64, 1.0 + 1.0j, 0j, batch=3, bcast=bcast)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))


@pytest.mark.parametrize("bcast", [None, "b"])
def test_complex_batch_above_grid_z_limit(bcast, cuda):
    """70000 batch entries: the planar split, the real GEMMs and the combine all stride in z."""
    got, want, _, _ = _run_cx(True, (0, 1), 2, 3, 4, 0.5 - 1.0j, 0.25 + 0.5j, batch=70000,
                              bcast=bcast)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
    got, want, _, _ = _run_cx(False, (1, 0), 2, 3, 4, 0.5 - 1.0j, 0.25 + 0.5j, batch=70000,
                              bcast=bcast, path=vk.PATH_SIMT)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_c64_default_path_accuracy(cuda):
    """512^3: the four fp32 GEMMs take the default (3xTF32) path."""
    got, want, C0, (ldc, sc, batch, M, N) = _run_cx(False, (0, 0), 512, 512, 512, 0.5 - 0.5j,
                                                     0.25 + 0j)
    g = got.view(np.complex64).reshape(M, ldc)
    w = want.view(np.complex64).reshape(M, ldc)
    err = np.linalg.norm(g[:, :N] - w[:, :N]) / np.linalg.norm(w[:, :N])
    assert err <= 1e-5, err
    assert np.array_equal(g[:, N:], C0.view(np.complex64).reshape(M, ldc)[:, N:])


# ---------------------------------------------------------- hipBLAS entry points
def _c(z, dt):
    return (dt * 2)(z.real, z.imag)


@pytest.mark.parametrize("trans", [(111, 111), (112, 111), (111, 112), (112, 112)],
                         ids=["NN", "TN", "NT", "TT"])
def test_hipblas_dgemm_cgemm_zgemm(trans, cuda):
    """Column-major hipBLAS calls equal the oracle of the swapped row-major
    problem (src/vkblas_hipblas.c:477-481, 544-548)."""
    import torch
    tA, tB = trans
    m, n, k = 45, 38, 70
    ta, tb = int(tA == 112), int(tB == 112)
    lda = (k if ta else m) + 2
    ldb = (n if tb else k) + 1
    ldc = m + 4
    na, nb, nc = (m if ta else k) * lda, (k if tb else n) * ldb, n * ldc
    rng = np.random.default_rng(tA + 2 * tB)
    with hb.Handle() as h:
        h.set_stream(torch.cuda.current_stream())
        # fp64
        A, B, C0 = rng.standard_normal(na), rng.standard_normal(nb), rng.standard_normal(nc)
        dA, dB, dC = _dev(A), _dev(B), _dev(C0)
        al, be = C.c_double(1.5), C.c_double(0.5)
        st = vk.lib.hipblasDgemm(h.h, tA, tB, m, n, k, C.byref(al), dA.data_ptr(), lda,
                                 dB.data_ptr(), ldb, C.byref(be), dC.data_ptr(), ldc)
        torch.cuda.synchronize()
        assert st == 0
        want = C0.copy()
        orc.dgemm_rowmajor_seq(tb, ta, n, m, k, 1.5, B, ldb, A, lda, 0.5, want, ldc)
        assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))
        # complex128 and complex64 (the latter on the exact path)
        for dbl in (True, False):
            dt = np.float64 if dbl else np.float32
            ct = C.c_double if dbl else C.c_float
            A, B, C0 = _cx(rng, na, dt), _cx(rng, nb, dt), _cx(rng, nc, dt)
            dA, dB, dC = _dev(A), _dev(B), _dev(C0)
            alpha, beta = 0.5 + 1.0j, -0.25 + 0.75j
            vk.set_path(vk.PATH_SIMT)
            try:
                fn = vk.lib.hipblasZgemm_v2 if dbl else vk.lib.hipblasCgemm_v2
                st = fn(h.h, tA, tB, m, n, k, _c(alpha, ct), dA.data_ptr(), lda, dB.data_ptr(),
                        ldb, _c(beta, ct), dC.data_ptr(), ldc)
                torch.cuda.synchronize()
            finally:
                vk.set_path(vk.PATH_AUTO)
            assert st == 0
            want = C0.copy()
            (orc.zgemm_rowmajor if dbl else orc.cgemm_rowmajor)(tb, ta, n, m, k, alpha, B, ldb, A,
                                                                lda, beta, want, ldc)
            view = np.uint64 if dbl else np.uint32
            assert np.array_equal(dC.cpu().numpy().view(view), want.view(view))


def test_hipblas_zgemm_strided_batched_and_conjugate_forwarding(cuda):
    import torch
    m, n, k, batch = 30, 20, 40, 3
    rng = np.random.default_rng(9)
    lda, ldb, ldc = m, k, m
    sA, sB, sC = m * k, k * n, m * n
    A, B, C0 = _cx(rng, sA * batch, np.float64), _cx(rng, sB * batch, np.float64), _cx(rng, sC * batch, np.float64)
    dA, dB, dC = _dev(A), _dev(B), _dev(C0)
    alpha, beta = 1.0 - 0.5j, 0.5 + 0j
    with hb.Handle() as h:
        h.set_stream(torch.cuda.current_stream())
        st = vk.lib.hipblasZgemmStridedBatched_v2(h.h, 111, 111, m, n, k, _c(alpha, C.c_double),
                                                  dA.data_ptr(), lda, sA, dB.data_ptr(), ldb, sB,
                                                  _c(beta, C.c_double), dC.data_ptr(), ldc, sC,
                                                  batch)
        torch.cuda.synchronize()
        assert st == 0
        want = C0.copy()
        orc.zgemm_rowmajor(0, 0, n, m, k, alpha, B, ldb, A, lda, beta, want, ldc, batch, sB, sA, sC)
        assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))
        # HIPBLAS_OP_C on a complex operand: no conjugating kernel here, so the
        # call goes to the real library -- none on this machine: NOT_SUPPORTED.
        before = dC.cpu().numpy().copy()
        st = vk.lib.hipblasZgemm_v2(h.h, 113, 111, m, n, k, _c(alpha, C.c_double), dA.data_ptr(),
                                    k, dB.data_ptr(), ldb, _c(beta, C.c_double), dC.data_ptr(), ldc)
        torch.cuda.synchronize()
        assert st == vk.HIPBLAS_STATUS_NOT_SUPPORTED
        assert np.array_equal(dC.cpu().numpy(), before)
