"""Engine housekeeping on a GPU: per-stream scratch workspaces
(vkblas_b200_release_workspaces gives the memory back, and the next call on
that stream allocates it again) and the kernel-timing event hook
(vkblas_b200_set_kernel_events brackets a call's main kernel)."""
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


def _timed_call(path, n=2048):
    """(whole-call ms, bracketed-kernel ms) of one SGEMM n^3 on `path`."""
    import torch
    s = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(n, n, device="cuda", generator=g)
    B = torch.randn(n, n, device="cuda", generator=g)
    C = torch.empty(n, n, device="cuda")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for e in ev:
        e.record(s)                        # creates the CUDA events
    vk.set_path(path)
    try:
        vk.gemm_tensors(0, 0, n, n, n, 1.0, A, n, B, n, 0.0, C, n, stream=s)   # warm-up
        torch.cuda.synchronize()
        vk.set_kernel_events(ev[1], ev[2])
        ev[0].record(s)
        vk.gemm_tensors(0, 0, n, n, n, 1.0, A, n, B, n, 0.0, C, n, stream=s)
        ev[3].record(s)
        vk.set_kernel_events(None, None)
        torch.cuda.synchronize()
    finally:
        vk.set_kernel_events(None, None)
        vk.set_path(vk.PATH_AUTO)
    assert vk.last_path() == path
    return ev[0].elapsed_time(ev[3]), ev[1].elapsed_time(ev[2])


def test_kernel_events_bracket_the_main_kernel(cuda):
    # 3xTF32: split pre-pass, then the GEMM -- the hook brackets the GEMM only
    call_ms, kern_ms = _timed_call(vk.PATH_TC)
    assert 0.0 < kern_ms < call_ms
    # exact SIMT: one kernel, so the bracket is nearly the whole call
    call_ms, kern_ms = _timed_call(vk.PATH_SIMT)
    assert 0.0 < kern_ms <= call_ms
    assert kern_ms > 0.9 * call_ms
