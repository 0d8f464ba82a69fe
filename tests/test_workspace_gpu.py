"""Per-stream scratch workspaces: vkblas_b200_release_workspaces gives the
memory back, and the next call on that stream allocates it again."""
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402


def _sgemm(stream, n, seed):
    """3xTF32 SGEMM n^3 on `stream` (its operand planes live in the stream's
    workspace); returns the relative Frobenius error against fp64."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(n, n, device="cuda", generator=g)
    B = torch.randn(n, n, device="cuda", generator=g)
    C = torch.empty(n, n, device="cuda")
    torch.cuda.synchronize()
    vk.gemm_tensors(0, 0, n, n, n, 1.0, A, n, B, n, 0.0, C, n, stream=stream)
    torch.cuda.synchronize()
    assert vk.last_path() == vk.PATH_TC
    want = A.double() @ B.double()
    return (torch.linalg.norm(C.double() - want) / torch.linalg.norm(want)).item()


def test_release_one_stream_then_reuse(cuda):
    import torch
    n = 2048                    # planes: 4 x 2048^2 fp32 = 64 MiB on this stream
    s = torch.cuda.Stream()
    assert _sgemm(s, n, 1) <= 1e-5
    free0, _ = torch.cuda.mem_get_info()
    vk.release_workspaces(s)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 - free0 >= 64 << 20, (free0, free1)
    assert _sgemm(s, n, 2) <= 1e-5          # allocated again on demand
    free2, _ = torch.cuda.mem_get_info()
    assert free1 - free2 >= 64 << 20, (free1, free2)


def test_release_other_stream_keeps_mine(cuda):
    import torch
    n = 1024                    # 16 MiB of planes per stream
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    assert _sgemm(s1, n, 3) <= 1e-5
    assert _sgemm(s2, n, 4) <= 1e-5
    free0, _ = torch.cuda.mem_get_info()
    vk.release_workspaces(s1)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 - free0 >= 16 << 20
    free_before_s2, _ = torch.cuda.mem_get_info()
    assert _sgemm(s2, n, 5) <= 1e-5         # s2's workspace is still there: no allocation
    free_after_s2, _ = torch.cuda.mem_get_info()
    assert abs(free_after_s2 - free_before_s2) < (8 << 20)
    vk.release_workspaces(all_streams=True)
    free2, _ = torch.cuda.mem_get_info()
    assert free2 - free_after_s2 >= 16 << 20
