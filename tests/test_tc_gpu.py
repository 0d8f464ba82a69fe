"""tcgen05 tensor-core GEMM (forced path) against the double-precision oracle.

fp16 / bf16 (kind::f16, fp32 accumulate, RNE store): relative Frobenius error
<= 2e-3 (fp16) / 8e-3 (bf16, 8-bit mantissa output); fp32 (3xTF32):
<= 1e-5.  Every op combination, ragged M/N/K, alpha/beta, strided batches with
a broadcast operand, and a C with ldc > N whose padding must stay untouched.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import vkblas_b200 as vk  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from gpu_util import dev, host, dev_u16, host_u16, check_status  # noqa: E402

SHAPES = [
    (128, 256, 64),       # one tile, one k-block
    (256, 512, 320),      # several tiles, ragged k-block count
    (200, 300, 136),      # ragged M, N, K
    (64, 48, 1000),       # partial tiles, long K
    (1024, 768, 512),     # many tiles (persistent loop, accumulator double-buffer)
]
TOL = {vk.DT_F16: 2e-3, vk.DT_BF16: 8e-3, vk.DT_F32: 1e-5}


def _mk(dtype, rng, n):
    x = rng.uniform(-1, 1, n).astype(np.float32)
    if dtype == vk.DT_F32:
        return x, None
    bits = orc.narrow(1 if dtype == vk.DT_BF16 else 0, x)
    return orc.widen(1 if dtype == vk.DT_BF16 else 0, bits), bits


def _run(dtype, op_a, op_b, M, N, K, alpha, beta, batch=1, bcast=None, ldc_pad=8, split=None,
         pair=None, tile_n=None):
    import torch
    rng = np.random.default_rng(M * 7 + N * 3 + K + op_a * 2 + op_b + dtype * 11 + batch)
    lda = (M if op_a else K)
    ldb = (K if op_b else N)
    if dtype != vk.DT_F32:      # 16-byte multiples for TMA
        lda = (lda + 7) // 8 * 8
        ldb = (ldb + 7) // 8 * 8
    else:
        lda += 1                # fp32 accepts any ld (the split pre-pass compacts)
        ldb += 3
    ldc = N + ldc_pad
    rows_a = K if op_a else M
    rows_b = N if op_b else K
    sa = 0 if bcast == "a" else rows_a * lda
    sb = 0 if bcast == "b" else rows_b * ldb
    sc = M * ldc
    na = (sa * (batch - 1) if sa else 0) + rows_a * lda
    nb = (sb * (batch - 1) if sb else 0) + rows_b * ldb
    nc = sc * (batch - 1) + M * ldc
    Af, Ab = _mk(dtype, rng, na)
    Bf, Bb = _mk(dtype, rng, nb)
    Cf, Cb = _mk(dtype, rng, nc)
    dt16 = 1 if dtype == vk.DT_BF16 else 0
    if dtype == vk.DT_F32:
        dA, dB, dC = dev(Af), dev(Bf), dev(Cf)
    else:
        dA, dB, dC = dev_u16(Ab, dt16), dev_u16(Bb, dt16), dev_u16(Cb, dt16)
    vk.set_path(vk.PATH_TC)
    try:
        vk.set_stream(torch.cuda.current_stream())
        st = vk.gemm(dtype, op_a, op_b, M, N, K, alpha, dA.data_ptr(), lda, dB.data_ptr(), ldb,
                     beta, dC.data_ptr(), ldc, batch, sa, sb, sc)
        torch.cuda.synchronize()
    finally:
        vk.set_path(vk.PATH_AUTO)
    assert st == vk.VKBLAS_OK, f"status {st}"
    assert vk.last_path() == vk.PATH_TC
    if split is not None:
        assert (vk.last_split() > 1) == split, f"K-split count {vk.last_split()}"
    if pair is not None:
        assert vk.last_pair() == pair, f"CTA pair mode {vk.last_pair()}"
    if tile_n is not None:
        assert vk.last_tile_n() == tile_n, f"tile N {vk.last_tile_n()}"
    check_status()
    got = host(dC) if dtype == vk.DT_F32 else orc.widen(dt16, host_u16(dC))
    want = orc.gemm_rowmajor_f64(op_a, op_b, M, N, K, alpha, np.ascontiguousarray(Af), lda,
                                 np.ascontiguousarray(Bf), ldb, beta, np.ascontiguousarray(Cf), ldc,
                                 batch, sa, sb, sc)
    for bi in range(batch):
        g = got[bi * sc: bi * sc + M * ldc].reshape(M, ldc)
        err = orc.rel_frobenius(g[:, :N], want[bi])
        assert err <= TOL[dtype], f"batch {bi}: relative error {err}"
        pad = g[:, N:]
        c0 = Cf[bi * sc: bi * sc + M * ldc].reshape(M, ldc)[:, N:]
        np.testing.assert_array_equal(pad, c0)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_BF16, vk.DT_F32], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("ops", [(0, 0), (0, 1), (1, 0), (1, 1)], ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_tc_gemm(dtype, ops, shape, cuda):
    M, N, K = shape
    _run(dtype, ops[0], ops[1], M, N, K, 1.0, 0.0)


# Fewer tiles than SMs: each tile's K range is cut into splits whose fp32
# partials a second kernel adds in split order (split-K), when enough K work
# per tile is saved.  (shape, splits for 2-byte types, splits for fp32)
SPLIT_SHAPES = [
    ((256, 256, 4096), True, True),
    ((256, 384, 8192), True, True),
    ((200, 300, 6000), True, True),      # ragged M, N and K
    ((512, 512, 2048), False, True),     # too little K per tile to split fp16
    ((384, 640, 1024), False, True),
]


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_BF16, vk.DT_F32], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("ops", [(0, 0), (0, 1), (1, 0), (1, 1)], ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("case", SPLIT_SHAPES, ids=[f"{m}x{n}x{k}" for (m, n, k), _, _ in SPLIT_SHAPES])
def test_tc_gemm_split_k(dtype, ops, case, cuda):
    (M, N, K), split16, split32 = case
    _run(dtype, ops[0], ops[1], M, N, K, 1.25, 0.5,
         split=split32 if dtype == vk.DT_F32 else split16)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
def test_tc_split_k_batched_broadcast(dtype, cuda):
    _run(dtype, 0, 1, 192, 200, 4096, 1.0, -1.0, batch=2, bcast="b", split=True)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
def test_tc_split_k_tail(dtype, cuda):
    """More tiles than SMs (one tile per batch entry): whole waves run unsplit
    and only the last, partial wave is split along K (stream-K tail)."""
    if dtype == vk.DT_F32:
        _run(dtype, 0, 0, 64, 72, 1536, 1.0, 0.25, batch=150, split=True)
    else:
        _run(dtype, 1, 1, 64, 72, 4096, 0.5, 0.0, batch=149, split=True)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_BF16, vk.DT_F32], ids=["f16", "bf16", "f32"])
def test_tc_alpha_beta(dtype, cuda):
    _run(dtype, 0, 1, 192, 320, 256, 0.75, -0.5)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
@pytest.mark.parametrize("bcast", [None, "a", "b"])
def test_tc_batched(dtype, bcast, cuda):
    _run(dtype, 0, 0, 160, 136, 96, 1.0, 0.5, batch=3, bcast=bcast)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
def test_tc_split_k_graph_capture(dtype, cuda):
    """A split call (GEMM + programmatically dependent reduce) captured in a
    CUDA graph and replayed gives the eager call's result bit for bit."""
    import torch
    M, N, K = 256, 384, 8192
    tdt = torch.float32 if dtype == vk.DT_F32 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(M, K, device="cuda", generator=g).to(tdt)
    B = torch.randn(K, N, device="cuda", generator=g).to(tdt)
    C_eager = torch.zeros(M, N, device="cuda", dtype=tdt)
    C_graph = torch.zeros(M, N, device="cuda", dtype=tdt)
    s = torch.cuda.Stream()

    def call(C):
        st = vk.gemm(dtype, 0, 0, M, N, K, 0.5, A.data_ptr(), K, B.data_ptr(), N, 0.0,
                     C.data_ptr(), N)
        assert st == vk.VKBLAS_OK

    with torch.cuda.stream(s):
        vk.set_stream(s)
        call(C_eager)                       # sizes the workspace before capture
        torch.cuda.synchronize()
        assert vk.last_split() > 1
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            call(C_graph)
        for _ in range(2):
            C_graph.zero_()
            graph.replay()
    torch.cuda.synchronize()
    vk.set_stream(torch.cuda.current_stream())
    check_status()
    assert torch.equal(C_graph, C_eager)
    del graph


# Small-M 2-byte GEMMs (decode with up to 64 tokens, N >= 128) run transposed:
# C^T = op(B)^T op(A)^T with weight rows on the MMA's 128 lanes and the tokens
# on a 64-wide N tile; the epilogue writes C transposed.  (shape, split)
SMALL_M_SHAPES = [
    ((1, 4096, 512), False),
    ((7, 1000, 520), False),       # ragged N and K
    ((16, 384, 4096), True),       # 3 weight-row tiles: K split 16 ways
    ((33, 200, 136), False),
    ((64, 4096, 4096), True),      # 32 tiles: K split 4 ways
]


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("ops", [(0, 0), (0, 1), (1, 0), (1, 1)], ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("case", SMALL_M_SHAPES, ids=[f"{m}x{n}x{k}" for (m, n, k), _ in SMALL_M_SHAPES])
def test_tc_small_m_transposed(dtype, ops, case, cuda):
    (M, N, K), split = case
    _run(dtype, ops[0], ops[1], M, N, K, 0.75, -0.5, split=split)


def test_tc_small_m_batched_broadcast(cuda):
    _run(vk.DT_F16, 0, 1, 12, 640, 256, 1.0, 0.5, batch=3, bcast="b", split=False)


# 256-row tiles on 2-CTA clusters (tcgen05 cta_group::2: each CTA loads its
# 128 rows of A and half of the B tile) whenever M >= 256 and no K split is
# planned.  (shape, pair)
PAIR_SHAPES = [
    ((512, 512, 256), True),
    ((300, 520, 200), True),        # second pair tile: the other CTA has 44 rows
    ((384, 264, 200), True),        # the other CTA's rows entirely past M in tile 2
    ((1024, 768, 512), True),
    ((200, 300, 136), False),
]


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_BF16, vk.DT_F32], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("ops", [(0, 0), (0, 1), (1, 0), (1, 1)], ids=["NN", "NT", "TN", "TT"])
@pytest.mark.parametrize("case", PAIR_SHAPES, ids=[f"{m}x{n}x{k}" for (m, n, k), _ in PAIR_SHAPES])
def test_tc_cta_pair_tiles(dtype, ops, case, cuda):
    (M, N, K), pair = case
    _run(dtype, ops[0], ops[1], M, N, K, 0.5, 0.25, pair=pair)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
def test_tc_pair_tiles_with_split(dtype, cuda):
    """A pair tile split along K: each CTA publishes its 128-row half of the
    partial tile and the reduce kernel adds them per half."""
    _run(dtype, 0, 1, 256, 256, 4096, 1.0, 0.5, split=True, pair=True)


@pytest.mark.parametrize("dtype", [vk.DT_F16, vk.DT_F32], ids=["f16", "f32"])
def test_tc_pair_wave_tail_split(dtype, cuda):
    """75 pair tiles (one per batch entry) on 74 SM pairs: whole waves run
    unsplit, only the last pair tile is split along K."""
    _run(dtype, 0, 0, 256, 40, 4096, 1.0, 0.0, batch=75, split=True, pair=True)


_TAIL_SCRIPT = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import vkblas_b200 as vk
from oracle import oracle as orc
out = {}
check_oracle = sys.argv[3] == "1"
# dtype, op_a, op_b, M, N, K, batch, A and B broadcast: 1186 pair tiles -> 1184
# whole, 2 (batch entry 592) as halves; the second column tile holds columns
# 256-319, so its second half lies beyond N
for i, (dt, oa, ob, M, N, K, batch) in enumerate([
        (vk.DT_F16, 0, 0, 256, 320, 3584, 593),
        (vk.DT_BF16, 1, 1, 256, 320, 3584, 593)]):
    rng = np.random.default_rng(50 + i)
    kind = 1 if dt == vk.DT_BF16 else 0
    ra, ca = (K, M) if oa else (M, K)
    rb, cb = (N, K) if ob else (K, N)
    ldc = N + 8
    sa, sb, sc = 0, 0, M * ldc
    A = orc.narrow(kind, rng.uniform(-1, 1, ra * ca).astype(np.float32))
    B = orc.narrow(kind, rng.uniform(-1, 1, rb * cb).astype(np.float32))
    C = orc.narrow(kind, rng.uniform(-1, 1, sc * batch).astype(np.float32))
    tdt = torch.bfloat16 if kind else torch.float16
    d = [torch.from_numpy(x.view(np.int16)).cuda().view(tdt) for x in (A, B, C)]
    vk.set_stream(torch.cuda.current_stream())
    vk.set_path(vk.PATH_TC)
    st = vk.gemm(dt, oa, ob, M, N, K, 0.75, d[0].data_ptr(), ca, d[1].data_ptr(), cb, 0.5,
                 d[2].data_ptr(), ldc, batch, sa, sb, sc)
    torch.cuda.synchronize()
    assert st == vk.VKBLAS_OK and vk.last_path() == vk.PATH_TC and vk.last_pair(), (i, st)
    assert vk.device_status(True) == 0
    got = d[2].view(torch.int16).cpu().numpy().view(np.uint16)
    vals = orc.widen(kind, got)
    for b in ((0, batch - 1) if check_oracle else ()):   # a whole tile's entry and the tail's
        want = orc.hgemm_rowmajor_f64(kind, oa, ob, M, N, K, 0.75, A[b * sa:], ca, B[b * sb:], cb,
                                      0.5, C[b * sc:], ldc)[0]
        res = vals[b * sc: b * sc + M * ldc].reshape(M, ldc)[:, :N]
        err = orc.rel_frobenius(res, want)
        assert err <= (8e-3 if kind else 2e-3), (i, b, err)
    pad = np.stack([got[b * sc: b * sc + M * ldc].reshape(M, ldc)[:, N:] for b in range(batch)])
    pad0 = np.stack([C[b * sc: b * sc + M * ldc].reshape(M, ldc)[:, N:] for b in range(batch)])
    assert np.array_equal(pad, pad0), "ldc padding written"
    out[f"c{i}"] = got
np.savez(sys.argv[2], **out)
"""


def test_tc_narrow_tail_matches_whole_tiles(cuda, tmp_path):
    """The narrow tail (the last wave's tiles as two 256 x 128 halves, in a
    second grid launched as a programmatic dependent) against the same calls
    with whole tiles (VKBLAS_NARROW_TAIL=0 VKBLAS_TC_SPLIT=0: no K split
    either), each in its own process: within the oracle's tolerance, padding
    untouched, and bit for bit equal (the halves add the same products in the
    same k order)."""
    import os
    import subprocess
    import sys
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if sms != 148:
        pytest.skip("the tail shapes are chosen for 74 SM pairs")
    for dt, oa, ob, M, N, K, batch in ((vk.DT_F16, 0, 0, 256, 320, 3584, 593),
                                       (vk.DT_BF16, 1, 1, 256, 320, 3584, 593)):
        assert vk.tc_plan(dt, oa, ob, M, N, K, batch, num_sms=sms)["tail_tiles"] == 2
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = {}
    for flag in ("1", "0"):
        path = str(tmp_path / f"tail_{flag}.npz")
        r = subprocess.run([sys.executable, "-c", _TAIL_SCRIPT, root, path, flag],
                           capture_output=True,
                           text=True, timeout=300,
                           env=dict(os.environ, VKBLAS_NARROW_TAIL=flag, VKBLAS_TC_SPLIT=flag))
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[flag] = np.load(path)
    for k in res["1"].files:
        assert np.array_equal(res["1"][k], res["0"][k]), f"{k}: narrow tail differs from whole tiles"


@pytest.mark.parametrize("ops", [(0, 0), (1, 1)], ids=["NN", "TT"])
@pytest.mark.parametrize("split", [False, True], ids=["whole", "split"])
def test_tf32_wide_pair_tiles(ops, split, cuda):
    """fp32 GEMMs with M >= 256 and N >= 256 run on the 256 x 256 3xTF32 pair
    tiles (the headline's kernel), whole and with a split last wave."""
    M, N, K = (256, 256, 4096) if split else (512, 768, 256)
    _run(vk.DT_F32, ops[0], ops[1], M, N, K, 1.0, 0.5, split=split, pair=True, tile_n=256)


_NARROW_SCRIPT = """
import sys, numpy as np, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
import vkblas_b200 as vk
from oracle import oracle as orc
for (M, N, K), split in (((512, 768, 256), False), ((256, 256, 4096), True)):
    rng = np.random.default_rng(M + N + K)
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros(M * N, device="cuda")
    vk.set_stream(torch.cuda.current_stream())
    assert vk.gemm(vk.DT_F32, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0,
                   dC.data_ptr(), N) == vk.VKBLAS_OK
    torch.cuda.synchronize()
    assert vk.last_path() == vk.PATH_TC and vk.last_pair() and vk.last_tile_n() == 128, \
        (vk.last_path(), vk.last_pair(), vk.last_tile_n())
    assert (vk.last_split() > 1) == split, vk.last_split()
    want = orc.gemm_rowmajor_f64(0, 0, M, N, K, 1.0, A, K, B, N, 0.0, None, N)[0]
    err = orc.rel_frobenius(dC.cpu().numpy().reshape(M, N), want)
    assert err <= 1e-5, err
    assert vk.device_status(True) == 0
print("OK")
"""


def test_tf32_narrow_pair_tiles_when_wide_is_off(cuda):
    """VKBLAS_TF32_WIDE=0 keeps the 256 x 128 pair tiles for N >= 256 (read once
    per process, so in a child process), whole and split; oracle-checked."""
    import os
    import subprocess
    import sys
    tests = os.path.dirname(os.path.abspath(__file__))
    code = _NARROW_SCRIPT.format(root=os.path.dirname(tests), tests=tests)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, VKBLAS_TF32_WIDE="0"))
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr[-3000:]


def test_tf32_transposed_split_beyond_grid_y_limit(cuda):
    """K above 65535 * 64 with both fp32 operands MN-major (op_a = T, op_b = N,
    the shape of a weight gradient over millions of tokens): the transposing
    3xTF32 pre-pass strides over k tiles instead of needing a larger grid, so
    the tail beyond the first 65535 tiles reaches the planes.  Checked against
    a double-precision product (numpy; the C oracle is far slower at this K)."""
    import torch
    M = N = 32
    K = 65537 * 64
    rng = np.random.default_rng(17)
    A = rng.standard_normal(K * M, dtype=np.float32)      # A[k * M + m]
    B = rng.standard_normal(K * N, dtype=np.float32)      # B[k * N + n]
    dA, dB = dev(A), dev(B)
    dC = torch.zeros(M * N, dtype=torch.float32, device="cuda")
    vk.set_path(vk.PATH_TC)
    try:
        vk.set_stream(torch.cuda.current_stream())
        st = vk.gemm(vk.DT_F32, 1, 0, M, N, K, 1.0, dA.data_ptr(), M, dB.data_ptr(), N, 0.0,
                     dC.data_ptr(), N, 1, 0, 0, 0)
        torch.cuda.synchronize()
    finally:
        vk.set_path(vk.PATH_AUTO)
    assert st == vk.VKBLAS_OK, f"status {st}"
    assert vk.last_path() == vk.PATH_TC
    check_status()
    want = A.reshape(K, M).astype(np.float64).T @ B.reshape(K, N).astype(np.float64)
    err = orc.rel_frobenius(host(dC).reshape(M, N), want)
    assert err <= TOL[vk.DT_F32], f"relative error {err}"
