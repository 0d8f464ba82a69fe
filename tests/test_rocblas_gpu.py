"""rocblas_gemm_strided_batched_ex parity on a B200 (reference
src/vkblas_hipblas.c:893-955, the PyTorch-on-ROCm batched path).

Every case goes through the C ABI exactly as rocBLAS callers bind it
(column-major, m/n/k and ld in rocBLAS terms, int64 strides, rocblas_datatype
values) and is compared with the double-precision oracle of the same
column-major problem, computed as the engine's row-major call the shim makes
(op_a = transB, op_b = transA, M = n, N = m, A <- b, B <- a;
src/vkblas_hipblas.c:234-239):

* f16, bf16 and f32, all four transA/transB, a batch of 3, a broadcast A
  (strideA = 0), padded ldd whose padding rows must stay untouched, device
  pointer mode for one case; relative Frobenius error <= 2e-3 (f16), 8e-3
  (bf16), 1e-5 (f32);
* the in-place rule: c != d, ldc != ldd, strideC != strideD or a compute type
  other than f32_r is forwarded -- not_implemented without a real rocBLAS --
  and D is not touched.
"""
import itertools

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import hipblas as hb  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import check_status  # noqa: E402

ROC = {0: vk.ROCBLAS_F16, 1: vk.ROCBLAS_BF16, 2: vk.ROCBLAS_F32}
TOL = {0: 2e-3, 1: 8e-3, 2: 1e-5}
ROCBLAS_POINTER_MODE_DEVICE = 1


def _rand(kind, n, rng, scale=1.0):
    x = (rng.uniform(-1, 1, n) * scale).astype(np.float32)
    return x if kind == 2 else orc.narrow(kind, x)


def _dev(kind, arr):
    import torch
    if kind == 2:
        return torch.from_numpy(np.ascontiguousarray(arr)).cuda()
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
    return t.view(torch.bfloat16 if kind else torch.float16)


def _host(kind, t):
    import torch
    if kind == 2:
        return t.cpu().numpy()
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _want(kind, ta, tb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C0, ldc, sC, batch):
    """Column-major C (batch, n, m) through the row-major double oracle."""
    if kind == 2:
        return orc.gemm_rowmajor_f64(tb, ta, n, m, k, alpha, B, ldb, A, lda, beta, C0, ldc,
                                     batch, sB, sA, sC)
    return orc.hgemm_rowmajor_f64(kind, tb, ta, n, m, k, alpha, B, ldb, A, lda, beta, C0, ldc,
                                  batch, sB, sA, sC)


def _gather(kind, flat, n, m, ldc, sC, batch):
    x = flat if kind == 2 else orc.widen(kind, flat)
    out = np.empty((batch, n, m), np.float64)
    for b in range(batch):
        out[b] = x[b * sC: b * sC + n * ldc].reshape(n, ldc)[:, :m]
    return out


def _call(h, ta, tb, m, n, k, al, dA, kind, lda, sA, dB, ldb, sB, be, dC, ldc, sC, dD, ldd, sD,
          batch, comp=vk.ROCBLAS_F32):
    t = ROC[kind]
    return vk.lib.rocblas_gemm_strided_batched_ex(
        h.h, vk.ROCBLAS_OP_T if ta else vk.ROCBLAS_OP_N, vk.ROCBLAS_OP_T if tb else vk.ROCBLAS_OP_N,
        m, n, k, al, dA.data_ptr(), t, lda, sA, dB.data_ptr(), t, ldb, sB, be, dC.data_ptr(), t,
        ldc, sC, dD.data_ptr(), t, ldd, sD, batch, comp, 0, 0, 0)


@pytest.mark.parametrize("bcast", [False, True])
@pytest.mark.parametrize("ta,tb", list(itertools.product((0, 1), repeat=2)))
@pytest.mark.parametrize("kind", [0, 1, 2])
def test_rocblas_strided_batched_against_oracle(kind, ta, tb, bcast, cuda):
    import torch
    m, n, k, batch = 160, 144, 136, 3
    alpha, beta = 1.25, -0.5
    ra, ca = (k, m) if ta else (m, k)           # column-major op(A) storage: ca columns of ra rows
    rb, cb = (n, k) if tb else (k, n)
    lda, ldb, ldc = ra + 8, rb + 16, m + 8      # multiples of 8 elements: tensor-core eligible
    sA = 0 if bcast else lda * ca + 24
    sB = ldb * cb + 8
    sC = ldc * n + 40
    rng = np.random.default_rng(1000 * kind + 100 * ta + 10 * tb + int(bcast))
    A = _rand(kind, (sA * (batch - 1) if sA else 0) + lda * ca, rng)
    B = _rand(kind, sB * (batch - 1) + ldb * cb, rng)
    C0 = _rand(kind, sC * batch, rng)
    dA, dB, dC = _dev(kind, A), _dev(kind, B), _dev(kind, C0)
    device_scalars = kind == 0 and ta == 1 and tb == 0 and not bcast
    with hb.RocHandle() as h:
        h.set_stream(torch.cuda.current_stream())
        if device_scalars:
            assert vk.lib.rocblas_set_pointer_mode(h.h, ROCBLAS_POINTER_MODE_DEVICE) == 0
            scal = torch.tensor([alpha, beta], dtype=torch.float32, device="cuda")
            al, be = scal[0:1].data_ptr(), scal[1:2].data_ptr()
        else:
            al, be = hb.fptr(alpha), hb.fptr(beta)
        st = _call(h, ta, tb, m, n, k, al, dA, kind, lda, sA, dB, ldb, sB, be, dC, ldc, sC, dC,
                   ldc, sC, batch)
        torch.cuda.synchronize()
    assert st == vk.rocblas_status_success
    check_status()
    assert vk.PATH_NAMES[vk.last_path()] == "tc", "expected the tensor-core path"
    want = _want(kind, ta, tb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C0, ldc, sC, batch)
    out = _host(kind, dC)
    got = _gather(kind, out, n, m, ldc, sC, batch)
    err = orc.rel_frobenius(got, want)
    assert err <= TOL[kind], f"relative error {err}"
    # padding rows of every column and the gaps between batch entries are untouched
    mask = np.ones(out.size, bool)
    for b in range(batch):
        idx = b * sC + np.arange(n)[:, None] * ldc + np.arange(m)[None, :]
        mask[idx.ravel()] = False
    assert np.array_equal(out[mask], C0[mask]), "D padding was written"


@pytest.mark.parametrize("kind", [0, 2])
def test_rocblas_strided_batched_ragged_ld_runs_exact_path(kind, cuda):
    """ld values TMA cannot describe (odd element counts) run on the SIMT kernel."""
    import torch
    m, n, k, batch = 37, 29, 45, 2
    lda, ldb, ldc = m + 3, k + 1, m + 5
    sA, sB, sC = lda * k + 1, ldb * n + 3, ldc * n + 7
    rng = np.random.default_rng(77 + kind)
    A, B, C0 = _rand(kind, sA * batch, rng), _rand(kind, sB * batch, rng), _rand(kind, sC * batch, rng)
    dA, dB, dC = _dev(kind, A), _dev(kind, B), _dev(kind, C0)
    al, be = hb.fptr(0.75), hb.fptr(0.25)
    with hb.RocHandle() as h:
        h.set_stream(torch.cuda.current_stream())
        st = _call(h, 0, 0, m, n, k, al, dA, kind, lda, sA, dB, ldb, sB, be, dC, ldc, sC, dC, ldc,
                   sC, batch)
        torch.cuda.synchronize()
    assert st == vk.rocblas_status_success
    assert vk.PATH_NAMES[vk.last_path()] == "simt"
    want = _want(kind, 0, 0, m, n, k, 0.75, A, lda, sA, B, ldb, sB, 0.25, C0, ldc, sC, batch)
    got = _gather(kind, _host(kind, dC), n, m, ldc, sC, batch)
    assert orc.rel_frobenius(got, want) <= (2e-3 if kind == 0 else 1e-6)
    if kind == 2:
        # the exact kernel is the reference's sequential-fmaf fp32 contract, bit for bit
        R = C0.copy()
        orc.gemm_rowmajor_f32seq(0, 0, n, m, k, 0.75, B, ldb, A, lda, 0.25, R, ldc, batch, sB, sA,
                                 sC)
        assert np.array_equal(_host(kind, dC).view(np.uint32), R.view(np.uint32))


def test_rocblas_strided_batched_inplace_rule(cuda):
    """Not in place, or compute type other than f32_r: forwarded (not_implemented
    here) and D untouched (src/vkblas_hipblas.c:904-908)."""
    import torch
    kind, m, n, k, batch = 0, 64, 64, 64, 2
    rng = np.random.default_rng(5)
    A, B = _rand(kind, m * k * batch, rng), _rand(kind, k * n * batch, rng)
    C0 = _rand(kind, m * n * batch * 2, rng)
    dA, dB, dC = _dev(kind, A), _dev(kind, B), _dev(kind, C0)
    dD = _dev(kind, np.full(C0.size, 0x3C00, np.uint16))           # 1.0 everywhere
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    s = m * n
    with hb.RocHandle() as h:
        h.set_stream(torch.cuda.current_stream())
        cases = [
            dict(dD=dD, ldd=m, sD=s),                      # c != d
            dict(dD=dC, ldd=m + 8, sD=s),                  # ldc != ldd
            dict(dD=dC, ldd=m, sD=2 * s),                  # strideC != strideD
            dict(dD=dC, ldd=m, sD=s, comp=vk.ROCBLAS_F16),   # compute type
        ]
        for c in cases:
            st = _call(h, 0, 0, m, n, k, al, dA, kind, m, s, dB, k, s, be, dC, m, s, c["dD"],
                       c["ldd"], c["sD"], batch, c.get("comp", vk.ROCBLAS_F32))
            torch.cuda.synchronize()
            assert st == vk.rocblas_status_not_implemented, c
    assert np.array_equal(_host(kind, dC), C0)
    assert (_host(kind, dD) == 0x3C00).all()
