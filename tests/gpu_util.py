"""Helpers shared by the GPU parity tests (imported only by tests marked gpu)."""
from __future__ import annotations

import ctypes as C

import numpy as np

import vkblas_b200 as vk
from vkblas_b200 import hipblas as hb
from oracle import oracle as orc


def dev(arr: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def host(t) -> np.ndarray:
    return t.cpu().numpy()


def dev_u16(arr: np.ndarray, dtype: int):
    """uint16 bit patterns -> a torch fp16/bf16 CUDA tensor with the same bits."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
    return t.view(torch.bfloat16 if dtype else torch.float16)


def host_u16(t) -> np.ndarray:
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def check_status(clear=True):
    st = vk.device_status(clear)
    assert st == 0, f"device status word {st}"


def sgemm_hip(h, c, dA, dB, dC, batched=False):
    a = hb.fptr(c["alpha"])
    b = hb.fptr(c["beta"])
    opA = vk.HIPBLAS_OP_T if c["ta"] else vk.HIPBLAS_OP_N
    opB = vk.HIPBLAS_OP_T if c["tb"] else vk.HIPBLAS_OP_N
    if not batched:
        return vk.lib.hipblasSgemm(h.h, opA, opB, c["m"], c["n"], c["k"], a, dA.data_ptr(), c["lda"],
                                   dB.data_ptr(), c["ldb"], b, dC.data_ptr(), c["ldc"])
    return vk.lib.hipblasSgemmStridedBatched(h.h, opA, opB, c["m"], c["n"], c["k"], a,
                                             dA.data_ptr(), c["lda"], c["sa"], dB.data_ptr(),
                                             c["ldb"], c["sb"], b, dC.data_ptr(), c["ldc"], c["sc"],
                                             c["batch"])


def colmajor_rows_ref(c, A, B, C0, rows):
    """Oracle (ref_gemm restatement) on the sampled rows: (batch, rows, n)."""
    batch = c.get("batch", 1)
    n, k, lda, ldc = c["n"], c["k"], c["lda"], c["ldc"]
    Cr = C0.copy()
    out = np.empty((batch, len(rows), n), np.float32)
    for b in range(batch):
        oA = c["sa"] * b if c.get("sa", 0) > 0 else 0
        oB = c["sb"] * b if c.get("sb", 0) > 0 else 0
        oC = c["sc"] * b if c.get("sc", 0) > 0 else 0
        Bb = np.ascontiguousarray(B[oB:])
        for ri, i in enumerate(rows):
            Ai = np.ascontiguousarray(A[oA + (i * lda if c["ta"] else i):])
            Ci = np.ascontiguousarray(Cr[oC + i:])
            orc.sgemm_colmajor_f64acc(c["ta"], c["tb"], 1, n, k, c["alpha"], Ai, lda, Bb,
                                      c["ldb"], c["beta"], Ci, ldc)
            out[b, ri, :] = Ci[np.arange(n) * ldc]
    return out


def gather_rows(c, Cflat, rows):
    batch = c.get("batch", 1)
    n, ldc = c["n"], c["ldc"]
    out = np.empty((batch, len(rows), n), np.float32)
    for b in range(batch):
        oC = c["sc"] * b if c.get("sc", 0) > 0 else 0
        for ri, i in enumerate(rows):
            out[b, ri, :] = Cflat[oC + i + np.arange(n) * ldc]
    return out
