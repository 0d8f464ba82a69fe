"""Case tables of the reference's own GEMM tests, restated as data.

The shapes, leading dimensions, alpha/beta, batch strides and seeds below are
the reference's test vectors (they are interface data and must be identical to
pin parity):

* ``TEST_GEMM_CASES`` / ``TEST_GEMM_BATCH_CASES`` -- test/test_gemm.c:226-293
  (hipBLAS column-major ``hipblasSgemm`` / ``hipblasSgemmStridedBatched``).
* ``TEST_H_CASES`` / ``TEST_H_BATCH_CASES`` -- test/test_h.c:89-105, 161-176
  (row-major engine ``vkblas_gemm_f16`` / ``vkblas_gemm_bf16``).
* ``TEST_V9H_CASES`` -- test/test_v9h.c:63-71 (through ``hipblasGemmEx``).
"""

# (m, n, k) list of test/test_gemm.c:227-232
_GEMM_SHAPES = [
    (32, 32, 32), (64, 64, 64), (128, 128, 128), (257, 129, 64), (100, 200, 300),
    (256, 256, 4096), (512, 512, 4096), (512, 640, 4096), (512, 768, 4096),
    (4096, 4096, 4096), (4096, 1024, 4096), (1024, 4096, 4096), (512, 512, 512),
    (33, 65, 17), (1, 64, 64), (64, 1, 64), (3, 5, 7),
]


def _gemm_cases():
    out = []
    for s, (m, n, k) in enumerate(_GEMM_SHAPES):
        for ta in (0, 1):
            for tb in (0, 1):
                lda = k if ta else m
                ldb = n if tb else k
                ldc = m
                out.append(dict(name=f"{'T' if ta else 'N'}{'T' if tb else 'N'} {m}x{n}x{k}",
                                ta=ta, tb=tb, m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc,
                                alpha=1.0, beta=0.0, seed=42 + s * 10 + ta * 2 + tb))
    # test/test_gemm.c:251-256
    out.append(dict(name="alpha=0.5 beta=0.7", ta=1, tb=1, m=256, n=128, k=64, lda=64, ldb=128,
                    ldc=256, alpha=0.5, beta=0.7, seed=7))
    out.append(dict(name="padded lda=140 ldb=80 ldc=300", ta=0, tb=1, m=128, n=64, k=64, lda=140,
                    ldb=80, ldc=300, alpha=1.0, beta=0.0, seed=8))
    out.append(dict(name="padded both T", ta=1, tb=1, m=100, n=50, k=80, lda=120, ldb=90, ldc=150,
                    alpha=1.0, beta=1.0, seed=9))
    return out


TEST_GEMM_CASES = _gemm_cases()

# test/test_gemm.c:262-268: m, n, k, lda, ldb, ldc, sa, sb, sc, batch
_BATCH_SHAPES = [
    (64, 64, 64, 64, 64, 64, 4096, 4096, 4096, 8),
    (128, 128, 128, 128, 128, 128, 16384, 16384, 16384, 6),
    (256, 256, 256, 256, 256, 256, 65536, 65536, 65536, 4),
    (33, 65, 17, 40, 70, 40, 2800, 1190, 2600, 5),
    (100, 200, 300, 320, 310, 110, 32000, 62000, 22000, 3),
]


def _gemm_batch_cases():
    out = []
    for s, (m, n, k, lda, ldb, ldc, sa, sb, sc, b) in enumerate(_BATCH_SHAPES):
        for ta in (0, 1):
            for tb in (0, 1):
                out.append(dict(name=f"{'T' if ta else 'N'}{'T' if tb else 'N'} {m}x{n}x{k}",
                                ta=ta, tb=tb, m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc,
                                sa=sa, sb=sb, sc=sc, batch=b, alpha=1.0, beta=0.0,
                                seed=100 + s * 10 + ta * 2 + tb))
    # test/test_gemm.c:285-293
    out.append(dict(name="alpha=0.5 beta=0.7 b=4", ta=0, tb=0, m=64, n=64, k=64, lda=64, ldb=64,
                    ldc=64, sa=4096, sb=4096, sc=4096, batch=4, alpha=0.5, beta=0.7, seed=7))
    out.append(dict(name="broadcast strideA=0", ta=0, tb=0, m=96, n=48, k=32, lda=96, ldb=32,
                    ldc=96, sa=0, sb=1536, sc=4608, batch=6, alpha=1.0, beta=0.0, seed=8))
    out.append(dict(name="broadcast strideB=0", ta=1, tb=1, m=48, n=96, k=32, lda=32, ldb=96,
                    ldc=48, sa=1536, sb=0, sc=4608, batch=6, alpha=1.0, beta=1.0, seed=9))
    return out


TEST_GEMM_BATCH_CASES = _gemm_batch_cases()

# test/test_h.c:89
_H_SHAPES = [(4, 4, 4), (8, 4, 6), (64, 64, 64), (33, 65, 17), (128, 128, 128), (257, 129, 64),
             (64, 1, 64)]


def _h_cases():
    out = []
    for dt in (0, 1):
        for op_a in (0, 1):
            for op_b in (0, 1):
                for s, (M, N, K) in enumerate(_H_SHAPES):
                    lda = K + (M % 2)
                    ldb = (K if op_b else N) + (N % 2)
                    ldc = N + (K % 2)
                    ba = ((K if op_a else M) - 1) * lda + (M if op_a else K)
                    bb = ((N if op_b else K) - 1) * ldb + (K if op_b else N)
                    bc = (M - 1) * ldc + N
                    out.append(dict(dtype=dt, op_a=op_a, op_b=op_b, M=M, N=N, K=K, lda=lda,
                                    ldb=ldb, ldc=ldc, na=ba, nb=bb, nc=bc, alpha=1.0, beta=0.5,
                                    seed=0x5EED + (s + 7 * (op_b + 2 * (op_a + 2 * dt)))))
    return out


TEST_H_CASES = _h_cases()

# test/test_h.c:161-176
_HB_SHAPES = [(64, 64, 64), (128, 128, 128), (96, 48, 32)]


def _h_batch_cases():
    out = []
    NB = 4
    for dt in (0, 1):
        for op_a in (0, 1):
            for op_b in (0, 1):
                for s, (M, N, K) in enumerate(_HB_SHAPES):
                    lda, ldb, ldc = K, (K if op_b else N), N
                    ba1 = ((K if op_a else M) - 1) * lda + (M if op_a else K)
                    bb1 = ((N if op_b else K) - 1) * ldb + (K if op_b else N)
                    bc1 = (M - 1) * ldc + N
                    sa = lda * (K if op_a else M)
                    sb = ldb * (N if op_b else K)
                    sc = ldc * M
                    out.append(dict(dtype=dt, op_a=op_a, op_b=op_b, M=M, N=N, K=K, lda=lda,
                                    ldb=ldb, ldc=ldc, sa=sa, sb=sb, sc=sc, batch=NB,
                                    na=ba1 + sa * (NB - 1), nb=bb1 + sb * (NB - 1),
                                    nc=bc1 + sc * (NB - 1), alpha=1.0, beta=0.5,
                                    seed=0xBEEF + (s + 7 * (op_b + 2 * (op_a + 2 * dt)))))
    return out


TEST_H_BATCH_CASES = _h_batch_cases()

# test/test_v9h.c:63-71: row-major M, N, K, lda, ldb, ldc, ta, tb (all N, ldc even)
TEST_V9H_CASES = [
    (256, 256, 256, 256, 256, 256, 0, 1),
    (130, 258, 70, 74, 72, 260, 0, 1),
    (256, 256, 256, 256, 256, 256, 1, 0),
    (130, 258, 70, 130, 258, 260, 1, 0),
    (130, 258, 70, 74, 260, 260, 0, 0),
    (256, 512, 256, 256, 512, 512, 0, 1),
    (64, 64, 48, 48, 64, 64, 0, 1),
]


def gemm_sizes(c):
    """Element counts of A, B, C for a test_gemm case (test/test_gemm.c:65-67, 136-141)."""
    szA1 = c["lda"] * (c["m"] if c["ta"] else c["k"])
    szB1 = c["ldb"] * (c["k"] if c["tb"] else c["n"])
    szC1 = c["ldc"] * c["n"]
    b = c.get("batch", 1)
    szA = (c["sa"] * (b - 1) if c.get("sa", 0) > 0 else 0) + szA1
    szB = (c["sb"] * (b - 1) if c.get("sb", 0) > 0 else 0) + szB1
    szC = (c["sc"] * (b - 1) if c.get("sc", 0) > 0 else 0) + szC1
    return szA, szB, szC


def sample_rows(m, n, k):
    """Row sampling of test/test_gemm.c:36-43, 87: 12 rows when m*n*k > 5e6."""
    if m * n * k <= 5_000_000:
        return list(range(m))
    s = 12
    if s >= m:
        return list(range(m))
    rows = [(r * m) // s for r in range(s)]
    rows[-1] = m - 1
    return rows
