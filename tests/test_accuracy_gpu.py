"""Error growth with K of the fp32 paths (B200), against a double-precision GEMM.

The tensor core's fp32 accumulation truncates: a 3xTF32 GEMM that keeps one
accumulator per tile has a relative error that grows ~7e-9 * K, biased toward
zero.  The 3xTF32 kernel accumulates 256-wide K segments separately and adds
them with round-to-nearest, so its error must stay flat in K and under the
1e-5 relative-Frobenius bar; the exact FFMA kernel is the yardstick.  Run with
-s to print the table (profiles/sgemm_3xtf32_accuracy.md).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402


@pytest.mark.parametrize("dist", ["normal", "test_gemm"])
def test_3xtf32_error_is_flat_in_k(dist, cuda):
    import torch
    vk.set_stream(torch.cuda.current_stream())
    M = N = 512
    errs = {}
    for K in (256, 1024, 4096, 16384):
        rng = np.random.default_rng(K)
        if dist == "normal":
            A = rng.standard_normal(M * K).astype(np.float32)
            B = rng.standard_normal(K * N).astype(np.float32)
        else:     # the value set of test/test_gemm.c:71-73
            A = (rng.integers(-100, 100, M * K) / 10).astype(np.float32)
            B = (rng.integers(-100, 100, K * N) / 10).astype(np.float32)
        want = orc.gemm_rowmajor_f64(0, 0, M, N, K, 1.0, A, K, B, N, 0.0, None, N)[0]
        row = []
        for name, path in (("3xtf32", vk.PATH_TC), ("ffma", vk.PATH_SIMT)):
            dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
            dC = torch.zeros(M * N, device="cuda")
            vk.set_path(path)
            try:
                st = vk.gemm(vk.DT_F32, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0,
                             dC.data_ptr(), N)
                torch.cuda.synchronize()
            finally:
                vk.set_path(vk.PATH_AUTO)
            assert st == vk.VKBLAS_OK
            got = dC.cpu().numpy().reshape(M, N).astype(np.float64)
            e = got - want
            rel = orc.rel_frobenius(got, want)
            bias = float(np.mean(e * np.sign(want)) / max(np.mean(np.abs(e)), 1e-300))
            row.append(f"{name}: relF={rel:.2e} max|d|={np.abs(e).max():.3e} bias={bias:+.2f}")
            errs[(name, K)] = rel
        print(f"{dist:9s} K={K:6d} |C|max={np.abs(want).max():9.1f}  " + "  ".join(row))
    for K in (256, 1024, 4096, 16384):
        assert errs[("3xtf32", K)] <= 1e-5
    # flat in K: the largest K is no worse than 2x the smallest
    assert errs[("3xtf32", 16384)] <= 2 * errs[("3xtf32", 256)] + 1e-7
