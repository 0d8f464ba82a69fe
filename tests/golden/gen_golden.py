"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run where the reference tree exists (it builds ``oracle/_ref`` from it):

    VKBLAS_REFERENCE_DIR=/path/to/vkblas python tests/golden/gen_golden.py

Outputs (committed, about 1 MB):

* ``ref_test_gemm.npz`` -- for every case of test/test_gemm.c:226-293 (single
  and strided-batched): sha256 of the inputs as test/test_gemm.c:70-73 makes
  them, and the output of the reference's own ``ref_gemm``
  (test/test_gemm.c:32-58) on the rows that test samples.  Small cases keep the
  full output array; large ones keep its sha256 plus the first sampled row.
* ``ref_test_h.npz`` -- for every case of test/test_h.c:89-226: sha256 of the
  inputs built with libc ``rand`` and the reference's own encoders
  (test/test_h.c:16-41), and the reference ``cpu_ref`` output
  (test/test_h.c:63-79): the array for small cases, its sha256 for all.

The inputs are drawn here twice: once through glibc ``rand`` called from
Python with the reference's compiled encoders, once through the oracle's C
generator; the script refuses to write fixtures when the two disagree.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as orc  # noqa: E402
import ref_cases as rc  # noqa: E402

libc = ctypes.CDLL("libc.so.6")
libc.rand.restype = ctypes.c_int
RAND_MAX = 2147483647


def sha(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def py_gen_test_gemm(seed, na, nb, nc):
    libc.srand(seed)
    out = []
    for n in (na, nb, nc):
        v = np.array([(libc.rand() % 200 - 100) for _ in range(n)], np.int64)
        out.append((v.astype(np.float32) / np.float32(10.0)).astype(np.float32))
    return out


def py_gen_test_h(seed, dtype, na, nb, nc, batched):
    ref = orc.ref
    libc.srand(seed)

    def uni():
        return np.float32(np.float32(libc.rand()) / np.float32(RAND_MAX) * np.float32(2.0) - np.float32(1.0))

    A = np.empty(na, np.uint16)
    B = np.empty(nb, np.uint16)
    C = np.empty(nc, np.uint16)
    for arr in (A, B, C):
        for i in range(arr.size):
            arr[i] = ref.vkref_f2h(float(uni()) if (dtype == 0 or batched) else 0.0)
    if dtype:
        for arr in (A, B, C):
            for i in range(arr.size):
                arr[i] = ref.vkref_f2bf(float(uni()))
    return A, B, C


def main() -> None:
    orc.build()
    import importlib
    importlib.reload(orc)
    if orc.ref is None:
        raise SystemExit("oracle/_ref/libvkref.so missing: the reference tree is needed")
    ref = orc.ref

    # ---------------------------------------------------------- test_gemm
    rec = {}
    cases = [("single", c) for c in rc.TEST_GEMM_CASES] + [("batch", c) for c in rc.TEST_GEMM_BATCH_CASES]
    for idx, (kind, c) in enumerate(cases):
        na, nb, nc = rc.gemm_sizes(c)
        A, B, C0 = orc.gen_test_gemm(c["seed"], na, nb, nc)
        if na + nb + nc <= 200_000:
            pA, pB, pC = py_gen_test_gemm(c["seed"], na, nb, nc)
            assert sha(A, B, C0) == sha(pA, pB, pC), f"generator mismatch on case {c['name']}"
        m, n, k = c["m"], c["n"], c["k"]
        rows = rc.sample_rows(m, n, k)
        sample = 12 if len(rows) < m else 0
        Cr = C0.copy()
        batch = c.get("batch", 1)
        for b in range(batch):
            offA = c["sa"] * b if c.get("sa", 0) > 0 else 0
            offB = c["sb"] * b if c.get("sb", 0) > 0 else 0
            offC = c["sc"] * b if c.get("sc", 0) > 0 else 0
            Ab = np.ascontiguousarray(A[offA:])
            Bb = np.ascontiguousarray(B[offB:])
            Cb = np.ascontiguousarray(Cr[offC:])
            ref.vkref_ref_gemm(c["ta"], c["tb"], m, n, k, c["alpha"], Ab, c["lda"], Bb, c["ldb"],
                               c["beta"], Cb, c["ldc"], sample)
            Cr[offC:] = Cb
        # gather the checked region: batches x sampled rows x n columns
        ldc = c["ldc"]
        out = np.empty((batch, len(rows), n), np.float32)
        for b in range(batch):
            offC = c["sc"] * b if c.get("sc", 0) > 0 else 0
            for ri, i in enumerate(rows):
                out[b, ri, :] = Cr[offC + i + np.arange(n) * ldc]
        key = f"g{idx:03d}"
        rec[key + "_kind"] = np.array(kind)
        rec[key + "_name"] = np.array(c["name"])
        rec[key + "_in_sha"] = np.array(sha(A, B, C0))
        rec[key + "_out_sha"] = np.array(sha(out))
        if out.size <= 4096:
            rec[key + "_out"] = out
        else:
            rec[key + "_out_row0"] = out[0, 0]
        print(f"{kind:6s} {c['name']:34s} rows={len(rows):5d} out={out.size}")
    np.savez_compressed(os.path.join(HERE, "ref_test_gemm.npz"), **rec)

    # ------------------------------------------------------------- test_h
    rec = {}
    hcases = [("single", c) for c in rc.TEST_H_CASES] + [("batch", c) for c in rc.TEST_H_BATCH_CASES]
    for idx, (kind, c) in enumerate(hcases):
        batched = kind == "batch"
        A, B, C0 = py_gen_test_h(c["seed"], c["dtype"], c["na"], c["nb"], c["nc"], batched)
        oA, oB, oC = orc.gen_test_h(c["seed"], c["dtype"], c["na"], c["nb"], c["nc"], batched)
        assert sha(A, B, C0) == sha(oA, oB, oC), f"test_h generator mismatch {c}"
        R = C0.copy()
        for b in range(c.get("batch", 1)):
            sa, sb, sc = c.get("sa", 0) * b, c.get("sb", 0) * b, c.get("sc", 0) * b
            Ab = np.ascontiguousarray(A[sa:])
            Bb = np.ascontiguousarray(B[sb:])
            Rb = np.ascontiguousarray(R[sc:])
            ref.vkref_cpu_ref_half(c["dtype"], c["op_a"], c["op_b"], c["M"], c["N"], c["K"], Ab,
                                   c["lda"], Bb, c["ldb"], c["alpha"], c["beta"], Rb, c["ldc"])
            R[sc:] = Rb
        key = f"h{idx:03d}"
        rec[key + "_kind"] = np.array(kind)
        rec[key + "_in_sha"] = np.array(sha(A, B, C0))
        rec[key + "_out_sha"] = np.array(sha(R))
        if R.size <= 4096:
            rec[key + "_R"] = R
    np.savez_compressed(os.path.join(HERE, "ref_test_h.npz"), **rec)
    print("wrote", len(hcases), "test_h cases")


if __name__ == "__main__":
    main()
