"""Seeded random GEMMs through the automatic path choice, and concurrent calls.

The shapes straddle every path boundary of the engine (GEMV for M <= 16 with
K-major weights, small-M transposed tcgen05 for M <= 64, single-CTA and CTA-pair
tiles around M = 256, K-splits, the exact SIMT kernel for small or misaligned
problems).  Each result is checked against the oracle with the bar of the
path that ran: bit-exact for SIMT fp32, 1e-5 for 3xTF32, 2e-3 / 8e-3 relative
for fp16 / bf16.  Padding columns of C must stay untouched.
"""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import check_status  # noqa: E402


def _cases(n=48, seed=2024):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        M = int(rng.choice([1, 3, 9, 16, 17, 40, 64, 65, 200, 255, 256, 300, 520]))
        N = int(rng.choice([8, 100, 128, 130, 257, 512, 700]))
        K = int(rng.choice([8, 24, 64, 200, 520, 1024, 2050]))
        dt = int(rng.choice([vk.DT_F32, vk.DT_F16, vk.DT_BF16]))
        op_a, op_b = int(rng.integers(2)), int(rng.integers(2))
        batch = int(rng.choice([1, 1, 1, 2, 3]))
        beta = float(rng.choice([0.0, 0.5, -1.0]))
        pad = int(rng.choice([0, 0, 8, 3]))
        out.append((i, M, N, K, dt, op_a, op_b, batch, beta, pad))
    return out


TOL = {vk.DT_F16: 2e-3, vk.DT_BF16: 8e-3}


def _run_case(M, N, K, dt, op_a, op_b, batch, beta, pad, seed, stream=None):
    import torch
    rng = np.random.default_rng(seed)
    lda = (M if op_a else K) + pad
    ldb = (K if op_b else N) + pad
    ldc = N + pad
    ra, rb = (K if op_a else M), (N if op_b else K)
    sa, sb, sc = ra * lda, rb * ldb, M * ldc
    na, nb, nc = sa * batch, sb * batch, sc * batch
    f = lambda n: rng.uniform(-1, 1, n).astype(np.float32)  # noqa: E731
    A, B, C0 = f(na), f(nb), f(nc)
    if dt != vk.DT_F32:
        d16 = 1 if dt == vk.DT_BF16 else 0
        Ab, Bb, Cb = orc.narrow(d16, A), orc.narrow(d16, B), orc.narrow(d16, C0)
        A, B, C0 = orc.widen(d16, Ab), orc.widen(d16, Bb), orc.widen(d16, Cb)
        tdt = torch.bfloat16 if d16 else torch.float16
        dA = torch.from_numpy(Ab.view(np.int16)).cuda().view(tdt)
        dB = torch.from_numpy(Bb.view(np.int16)).cuda().view(tdt)
        dC = torch.from_numpy(Cb.view(np.int16)).cuda().view(tdt)
    else:
        dA, dB, dC = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    s = stream or torch.cuda.current_stream()
    vk.set_stream(s)
    st = vk.gemm(dt, op_a, op_b, M, N, K, 0.75, dA.data_ptr(), lda, dB.data_ptr(), ldb, beta,
                 dC.data_ptr(), ldc, batch, sa, sb, sc)
    path = vk.last_path()
    s.synchronize()
    assert st == vk.VKBLAS_OK, st
    got = dC.float().cpu().numpy()
    if dt == vk.DT_F32 and path == vk.PATH_SIMT:
        want = C0.copy()
        orc.gemm_rowmajor_f32seq(op_a, op_b, M, N, K, 0.75, A, lda, B, ldb, beta, want, ldc, batch,
                                 sa, sb, sc)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "SIMT fp32 not exact"
        return path
    want = orc.gemm_rowmajor_f64(op_a, op_b, M, N, K, 0.75, A, lda, B, ldb, beta, C0, ldc, batch,
                                 sa, sb, sc)
    tol = 1e-5 if dt == vk.DT_F32 else TOL[dt]
    for b in range(batch):
        g = got[b * sc: b * sc + M * ldc].reshape(M, ldc)
        err = orc.rel_frobenius(g[:, :N], want[b])
        assert err <= tol, f"batch {b} path {vk.PATH_NAMES[path]}: relative error {err}"
        np.testing.assert_array_equal(g[:, N:], C0[b * sc: b * sc + M * ldc].reshape(M, ldc)[:, N:])
    return path


@pytest.mark.parametrize("case", _cases(), ids=lambda c: "r{}_{}x{}x{}_dt{}_{}{}_b{}".format(*c[:8]))
def test_random_auto_path(case, cuda):
    i, M, N, K, dt, op_a, op_b, batch, beta, pad = case
    _run_case(M, N, K, dt, op_a, op_b, batch, beta, pad, seed=1000 + i)
    check_status()


def test_concurrent_threads_on_own_streams(cuda):
    """Four host threads, each with its own stream, run random GEMMs at once:
    the per-thread path / stream state and the per-stream workspaces must keep
    them apart."""
    import torch
    cases = _cases(24, seed=7)
    errors = []

    def worker(tid):
        try:
            torch.cuda.set_device(0)
            s = torch.cuda.Stream()
            for j, c in enumerate(cases[tid::4]):
                _, M, N, K, dt, op_a, op_b, batch, beta, pad = c
                _run_case(M, N, K, dt, op_a, op_b, batch, beta, pad, seed=50 * tid + j, stream=s)
        except Exception as exc:        # reported on the main thread
            errors.append(f"thread {tid}: {exc!r}")

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(600)
    assert not errors, errors
    check_status()
