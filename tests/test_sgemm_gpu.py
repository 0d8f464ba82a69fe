"""fp32 GEMM parity through the hipBLAS ABI on a B200 (reference test/test_gemm.c).

Every shape, op combination, leading dimension, alpha/beta, batch stride and
seed of test/test_gemm.c:226-293 is run through ``hipblasSgemm`` /
``hipblasSgemmStridedBatched`` of libvkblas_hipblas.so and compared with the
oracle's restatement of the reference ``ref_gemm`` (pinned bit-for-bit to the
reference by tests/test_oracle.py) on the rows that test checks:

* reference bar (test/test_gemm.c:117): max |diff| < 0.1, every path;
* exact SIMT path: bit-identical to the sequential-fmaf oracle over the
  whole C array (padding included) wherever the oracle is cheap;
* 3xTF32 tensor-core path: relative Frobenius error <= 1e-5 against the
  double-accumulation oracle.
"""
import numpy as np
import pytest

import ref_cases as rc

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from vkblas_b200 import hipblas as hb  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev, host, sgemm_hip, colmajor_rows_ref, gather_rows, check_status  # noqa: E402

PATHS = {"simt": vk.PATH_SIMT, "auto": vk.PATH_AUTO}
SINGLE = rc.TEST_GEMM_CASES
BATCH = rc.TEST_GEMM_BATCH_CASES


@pytest.fixture(params=list(PATHS))
def path(request, cuda):
    vk.set_path(PATHS[request.param])
    yield request.param
    vk.set_path(vk.PATH_AUTO)


def _run_case(c, path, batched):
    import torch
    na, nb, nc = rc.gemm_sizes(c)
    A, B, C0 = orc.gen_test_gemm(c["seed"], na, nb, nc)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    n0 = vk.launch_count()
    with hb.Handle() as h:
        h.set_stream(torch.cuda.current_stream())
        st = sgemm_hip(h, c, dA, dB, dC, batched)
        torch.cuda.synchronize()
    assert st == vk.HIPBLAS_STATUS_SUCCESS
    assert vk.launch_count() > n0, "no kernel of libvkblas_hipblas.so ran"
    check_status()
    got = host(dC)
    rows = rc.sample_rows(c["m"], c["n"], c["k"])
    want = colmajor_rows_ref(c, A, B, C0, rows)
    g = gather_rows(c, got, rows)
    maxd = float(np.max(np.abs(g.astype(np.float64) - want)))
    assert maxd < 0.1, f"max|diff| {maxd} (reference bar 0.1)"
    ran = vk.last_path()
    if path == "simt":
        assert ran == vk.PATH_SIMT
    if ran == vk.PATH_SIMT and c["m"] * c["n"] * c["k"] * c.get("batch", 1) <= 6_000_000:
        ref = C0.copy()
        orc.gemm_rowmajor_f32seq(c["tb"], c["ta"], c["n"], c["m"], c["k"], c["alpha"], B, c["ldb"],
                                 A, c["lda"], c["beta"], ref, c["ldc"], c.get("batch", 1),
                                 c.get("sb", 0), c.get("sa", 0), c.get("sc", 0))
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    elif ran == vk.PATH_TC:
        err = orc.rel_frobenius(g, want)
        assert err <= 1e-5, f"3xTF32 relative Frobenius error {err}"
    # Nothing outside the stored C may change (padding rows of ldc, gaps between batches).
    mask = np.ones(nc, bool)
    for b in range(c.get("batch", 1)):
        oC = c["sc"] * b if c.get("sc", 0) > 0 else 0
        for j in range(c["n"]):
            mask[oC + j * c["ldc"]: oC + j * c["ldc"] + c["m"]] = False
    np.testing.assert_array_equal(got[mask], C0[mask])


@pytest.mark.parametrize("c", SINGLE, ids=[c["name"] for c in SINGLE])
def test_hipblas_sgemm_reference_cases(c, path):
    _run_case(c, path, batched=False)


@pytest.mark.parametrize("c", BATCH, ids=[c["name"] for c in BATCH])
def test_hipblas_sgemm_strided_batched_reference_cases(c, path):
    _run_case(c, path, batched=True)


def test_config1_1024_alpha_beta_all_ops(cuda):
    """1024^3, all four ops, ld=1024, alpha=1.5 beta=0.5,
    A/B/C uniform[-1,1] from seed; plus 3x5x7 and 64x1x64 with ld+3."""
    import torch
    rng = np.random.default_rng(1234)
    shapes = [(1024, 1024, 1024, 0), (3, 5, 7, 3), (64, 1, 64, 3)]
    for (m, n, k, pad) in shapes:
        for ta in (0, 1):
            for tb in (0, 1):
                lda = (k if ta else m) + pad
                ldb = (n if tb else k) + pad
                ldc = m + pad
                A = rng.uniform(-1, 1, lda * (m if ta else k)).astype(np.float32)
                B = rng.uniform(-1, 1, ldb * (k if tb else n)).astype(np.float32)
                C0 = rng.uniform(-1, 1, ldc * n).astype(np.float32)
                c = dict(ta=ta, tb=tb, m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc, alpha=1.5, beta=0.5)
                for p in (vk.PATH_SIMT, vk.PATH_AUTO):
                    vk.set_path(p)
                    dA, dB, dC = dev(A), dev(B), dev(C0)
                    with hb.Handle() as h:
                        st = sgemm_hip(h, c, dA, dB, dC)
                        torch.cuda.synchronize()
                    vk.set_path(vk.PATH_AUTO)
                    assert st == 0
                    got = host(dC)
                    want = C0.copy()
                    orc.sgemm_colmajor_f64acc(ta, tb, m, n, k, 1.5, A, lda, B, ldb, 0.5, want, ldc)
                    assert np.max(np.abs(got - want)) < 1e-2
                    assert orc.rel_frobenius(got, want) <= 1e-5
                    if p == vk.PATH_SIMT:
                        ref = C0.copy()
                        orc.gemm_rowmajor_f32seq(tb, ta, n, m, k, 1.5, B, ldb, A, lda, 0.5, ref, ldc)
                        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    check_status()


def test_device_pointer_mode(cuda):
    """alpha/beta in device memory: read by the kernel, no host round trip."""
    import torch
    rng = np.random.default_rng(7)
    m, n, k = 96, 80, 72
    A = rng.uniform(-1, 1, m * k).astype(np.float32)
    B = rng.uniform(-1, 1, k * n).astype(np.float32)
    C0 = rng.uniform(-1, 1, m * n).astype(np.float32)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    dal = torch.tensor([0.75], device="cuda")
    dbe = torch.tensor([-1.25], device="cuda")
    with hb.Handle() as h:
        assert vk.lib.hipblasSetPointerMode(h.h, vk.HIPBLAS_POINTER_MODE_DEVICE) == 0
        st = vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, m, n, k, dal.data_ptr(),
                                 dA.data_ptr(), m, dB.data_ptr(), k, dbe.data_ptr(), dC.data_ptr(), m)
        torch.cuda.synchronize()
    assert st == 0
    want = C0.copy()
    orc.sgemm_colmajor_f64acc(0, 0, m, n, k, 0.75, A, m, B, k, -1.25, want, m)
    assert np.max(np.abs(host(dC) - want)) < 1e-4


def test_beta_zero_does_not_read_c(cuda):
    """beta == 0: C is not read (src/vkblas.h:26) -- NaN garbage in C vanishes."""
    import torch
    rng = np.random.default_rng(8)
    m, n, k = 130, 66, 40
    A = rng.uniform(-1, 1, m * k).astype(np.float32)
    B = rng.uniform(-1, 1, k * n).astype(np.float32)
    for p in (vk.PATH_SIMT, vk.PATH_AUTO):
        C0 = np.full(m * n, np.nan, np.float32)
        dA, dB, dC = dev(A), dev(B), dev(C0)
        vk.set_path(p)
        vk.gemm_tensors(vk.OP_N, vk.OP_N, m, n, k, 1.0, dA, k, dB, n, 0.0, dC, n)
        torch.cuda.synchronize()
        vk.set_path(vk.PATH_AUTO)
        got = host(dC)
        assert np.isfinite(got).all()


def test_engine_rejects_bad_arguments(cuda):
    import torch
    x = torch.zeros(64, device="cuda")
    p = x.data_ptr()
    assert vk.gemm(vk.DT_F32, 0, 0, 0, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4) == vk.VKBLAS_ERR_PARAM
    assert vk.gemm(vk.DT_F32, 0, 0, 4, 4, 4, 1.0, 0, 4, p, 4, 0.0, p, 4) == vk.VKBLAS_ERR_PARAM
    assert vk.gemm(vk.DT_F32, 0, 0, 4, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4, batch=0) == vk.VKBLAS_ERR_PARAM
