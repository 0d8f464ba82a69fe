"""Host-side checks of the Python helpers (no GPU): gemm_tensors rejects
operands that do not fit the call before anything is launched."""
import pytest
import torch

import vkblas_b200 as vk


class FakeCuda:
    """Stands in for a CUDA tensor: only what the checks read."""

    def __init__(self, n, dtype=torch.float32, device="cuda:0", contiguous=True):
        self._n, self.dtype, self.device = n, dtype, torch.device(device)
        self.is_cuda, self._c = True, contiguous

    def numel(self):
        return self._n

    def is_contiguous(self):
        return self._c


def _check(*args, **kw):
    vk._check_tensors(*args, **kw)


def test_fitting_operands_pass():
    M, N, K = 5, 7, 3
    _check(0, 0, M, N, K, FakeCuda(M * K), K, FakeCuda(K * N), N, FakeCuda(M * N), N, 1, 0, 0, 0)
    # transposed operands, padded ld, a batch with a broadcast B
    _check(1, 1, M, N, K, FakeCuda(2 * K * (M + 1)), M + 1, FakeCuda(N * K), K,
           FakeCuda(2 * M * N), N, 2, K * (M + 1), 0, M * N)


@pytest.mark.parametrize("bad, msg", [
    (dict(A=torch.zeros(15)), "CUDA tensor"),
    (dict(B=FakeCuda(21, contiguous=False)), "contiguous"),
    (dict(C=FakeCuda(35, dtype=torch.float16)), "dtypes differ"),
    (dict(C=FakeCuda(35, device="cuda:1")), "devices differ"),
    (dict(A=FakeCuda(14)), "holds 14 elements"),
    (dict(lda=2), "lda = 2 < 3"),
    (dict(M=0), "positive"),
])
def test_bad_operands_raise(bad, msg):
    a = dict(M=5, N=7, K=3, A=FakeCuda(15), lda=3, B=FakeCuda(21), ldb=7, C=FakeCuda(35), ldc=7)
    a.update(bad)
    with pytest.raises(ValueError, match=msg):
        _check(0, 0, a["M"], a["N"], a["K"], a["A"], a["lda"], a["B"], a["ldb"], a["C"], a["ldc"],
               1, 0, 0, 0)


def test_gemm_tensors_rejects_host_tensors_before_any_launch():
    A, B, C = torch.zeros(6), torch.zeros(6), torch.zeros(4)
    with pytest.raises(ValueError, match="CUDA tensor"):
        vk.gemm_tensors(0, 0, 2, 2, 3, 1.0, A, 3, B, 2, 0.0, C, 2)
