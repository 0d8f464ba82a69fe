"""Run one GEMM case of the BASELINE configs a few times (for timing and ncu).

    python -m vkblas_b200.cases sgemm  [--n 4096] [--shape M,N,K] [--iters 3]   # 3xTF32, N/N
    python -m vkblas_b200.cases sgemm-simt [--n 4096]                # exact FFMA kernel
    python -m vkblas_b200.cases hgemm  [--n 4096] [--shape M,N,K]    # fp16 tcgen05, hipBLAS T/N
    python -m vkblas_b200.cases gemv   [--m 1] [--splitk 4]          # decode, K=4096, N=14336, M<=64
    python -m vkblas_b200.cases gemv32 [--m 1] [--trans t|n]         # fp32 decode, K=4096, N=14336
    python -m vkblas_b200.cases dgemm|zgemm [--n 2048]               # fp64 / complex128 N/N
    python -m vkblas_b200.cases batched                              # 256 x 2048^3 fp16 N/N

Inputs are device-resident and seeded; each iteration is one library call on
torch's current stream; the mean time per call (CUDA events) is printed.
--path simt|tc|gemv forces a kernel family (the call fails if it cannot run).
"""
from __future__ import annotations

import argparse

import torch

import vkblas_b200 as vk
from vkblas_b200 import hipblas as hb


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["sgemm", "sgemm-simt", "hgemm", "gemv", "gemv32", "batched",
                                     "dgemm", "zgemm"])
    ap.add_argument("--trans", default="t", choices=["t", "n"],
                    help="gemv32: hipBLAS transA of the weights (t: N x K rows, n: K x N)")
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--shape", default="", help="M,N,K (sgemm, sgemm-simt, hgemm); default n,n,n")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--splitk", type=int, default=0)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--path", default="auto", choices=["auto", "simt", "tc", "gemv"],
                    help="force a kernel family (vkblas_b200_set_path)")
    a = ap.parse_args(argv)

    torch.cuda.init()
    s = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(0)
    al, be = hb.fptr(1.0), hb.fptr(0.0)
    h = hb.Handle()
    h.set_stream(s)
    n = a.n
    M, N, K = (int(x) for x in a.shape.split(",")) if a.shape else (n, n, n)
    if a.case in ("sgemm", "sgemm-simt"):
        A = torch.randn(M * K, device="cuda", generator=g)
        B = torch.randn(K * N, device="cuda", generator=g)
        C = torch.empty(M * N, device="cuda")
        if a.case == "sgemm-simt":
            vk.set_path(vk.PATH_SIMT)
        flop, nbytes = 2.0 * M * N * K, 0.0
        # column-major C (M x N) = A (M x K) * B (K x N)
        call = lambda: vk.lib.hipblasSgemm(h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, M, N, K, al,  # noqa: E731
                                           A.data_ptr(), M, B.data_ptr(), K, be, C.data_ptr(), M)
    elif a.case == "hgemm":
        A = (torch.randn(M * K, device="cuda", generator=g) * 0.02).half()
        B = (torch.randn(K * N, device="cuda", generator=g) * 0.02).half()
        C = torch.empty(M * N, device="cuda", dtype=torch.float16)
        flop, nbytes = 2.0 * M * N * K, 0.0
        # column-major C (M x N) = A^T (A stored K x M) * B (K x N)
        call = lambda: vk.lib.hipblasGemmEx_v2(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, M, N, K, al,  # noqa: E731
                                               A.data_ptr(), vk.HIP_R_16F, K, B.data_ptr(),
                                               vk.HIP_R_16F, K, be, C.data_ptr(), vk.HIP_R_16F, M,
                                               vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
    elif a.case == "gemv":
        K, O, M = 4096, 14336, a.m
        # four weight sets (470 MB > 126 MB L2), rotated call by call
        Ws = [(torch.randn(O * K, device="cuda", generator=g) * 0.02).half() for _ in range(4)]
        X = torch.randn(M * K, device="cuda", generator=g).half()
        C = torch.empty(M * O, device="cuda", dtype=torch.float16)
        if a.splitk:
            vk.set_splitk(a.splitk)
        flop, nbytes = 2.0 * M * O * K, 2.0 * (O * K + M * K + M * O)
        turn = [0]

        def call():
            turn[0] += 1
            return vk.lib.hipblasGemmEx(h.h, vk.HIPBLAS_OP_T, vk.HIPBLAS_OP_N, O, M, K, al,
                                        Ws[turn[0] % 4].data_ptr(), vk.HIPBLAS_R_16F, K, X.data_ptr(),
                                        vk.HIPBLAS_R_16F, K, be, C.data_ptr(), vk.HIPBLAS_R_16F, O,
                                        vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)
    elif a.case == "gemv32":
        K, O, M = 4096, 14336, a.m
        # four fp32 weight sets (940 MB > 126 MB L2), rotated call by call
        Ws = [torch.randn(O * K, device="cuda", generator=g) * 0.02 for _ in range(4)]
        X = torch.randn(M * K, device="cuda", generator=g)
        C = torch.empty(M * O, device="cuda")
        if a.splitk:
            vk.set_splitk(a.splitk)
        flop, nbytes = 2.0 * M * O * K, 4.0 * (O * K + M * K + M * O)
        tA = vk.HIPBLAS_OP_T if a.trans == "t" else vk.HIPBLAS_OP_N
        lda = K if a.trans == "t" else O
        turn = [0]

        def call():
            turn[0] += 1
            return vk.lib.hipblasSgemm(h.h, tA, vk.HIPBLAS_OP_N, O, M, K, al,
                                       Ws[turn[0] % 4].data_ptr(), lda, X.data_ptr(), K, be,
                                       C.data_ptr(), O)
    elif a.case in ("dgemm", "zgemm"):
        cplx = a.case == "zgemm"
        w = 2 if cplx else 1
        A = torch.randn(w * M * K, device="cuda", generator=g, dtype=torch.float64)
        B = torch.randn(w * K * N, device="cuda", generator=g, dtype=torch.float64)
        C = torch.zeros(w * M * N, device="cuda", dtype=torch.float64)
        vk.set_stream(s)
        # useful FLOP: a complex multiply-add is 4 real ones
        flop, nbytes = (8.0 if cplx else 2.0) * M * N * K, 0.0
        if cplx:
            call = lambda: vk.lib.vkblas_gemm_z64(0, 0, M, N, K, 1.0, 0.0, A.data_ptr(), K,  # noqa: E731
                                                  B.data_ptr(), N, 0.0, 0.0, C.data_ptr(), N, 1,
                                                  0, 0, 0)
        else:
            call = lambda: vk.lib.vkblas_gemm_f64(0, 0, M, N, K, 1.0, A.data_ptr(), K,  # noqa: E731
                                                  B.data_ptr(), N, 0.0, C.data_ptr(), N, 1, 0, 0, 0)
    else:
        b, n = 256, 2048
        A = (torch.randn(b * n * n, device="cuda", generator=g) * 0.02).half()
        B = (torch.randn(b * n * n, device="cuda", generator=g) * 0.02).half()
        C = torch.empty(b * n * n, device="cuda", dtype=torch.float16)
        flop, nbytes = b * 2.0 * n ** 3, 0.0
        call = lambda: vk.lib.hipblasGemmStridedBatchedEx_v2(  # noqa: E731
            h.h, vk.HIPBLAS_OP_N, vk.HIPBLAS_OP_N, n, n, n, al, A.data_ptr(), vk.HIP_R_16F, n,
            n * n, B.data_ptr(), vk.HIP_R_16F, n, n * n, be, C.data_ptr(), vk.HIP_R_16F, n, n * n,
            b, vk.HIPBLAS_COMPUTE_32F, vk.HIPBLAS_GEMM_DEFAULT)

    if a.path != "auto":
        vk.set_path({"simt": vk.PATH_SIMT, "tc": vk.PATH_TC, "gemv": vk.PATH_GEMV}[a.path])
    st = call()
    if st != 0:
        raise SystemExit(f"status {st}")
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(a.iters):
        call()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, a.iters)
    st = vk.device_status(True)
    line = f"{a.case}: {ms * 1e3:.2f} us/call, {flop / ms / 1e9:.2f} TFLOP/s"
    if nbytes:
        line += f", {nbytes / ms / 1e6:.1f} GB/s"
    print(line + f", path={vk.PATH_NAMES[vk.last_path()]}, status={st}")
    h.close()
    return 0 if st == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
