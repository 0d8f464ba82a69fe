"""bench.py's reference arm (host CPU only) prints the one JSON line the driver
reads, with the keys its contract names."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--ref-seconds", "1"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "TFLOPS" and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_roofline_object_for_each_kernel_configuration():
    """The GPU arm's `roofline` object (built after the timed region, so a
    mistake there would cost the whole bench line) for the tile
    configurations the headline can run on: 256x256 pair tiles with a split
    last wave, 256x128 pair tiles, and the exact FFMA kernel; with the
    ceilings measured in the run and, when that measurement failed, with the
    peak derived from the bf16 burst."""
    sys.path.insert(0, ROOT)
    import bench
    peaks = {"hbm_gbs": 6548.2, "bf16_tflops": 1679.7, "sm_max_mhz": 1965.0}
    ceil = {"ffma_fp32": {"tflops": 71.7}, "tcgen05_tf32": {"tflops": 1112.6},
            "tcgen05_tf32_pair": {"tflops": 1111.0}, "tcgen05_f16": {"tflops": 2213.8},
            "tcgen05_f16_pair": {"tflops": 2059.7}}
    flop = 2.0 * 4096 ** 3
    gemm_ms, step_ms = 0.465, 0.548
    wide = bench._roofline("tc", 256, True, 2, gemm_ms, step_ms, peaks, "measured", ceil)
    assert wide["kernel"] == ("3xTF32 tcgen05 SGEMM (umma_gemm_kernel, 256x256 tiles on CTA "
                              "pairs; last wave split 2 ways, then split_reduce_kernel)")
    assert abs(wide["achieved"] - flop / gemm_ms / 1e9) < 0.01
    assert abs(wide["peak"] - 1111.0 / 3) < 0.01 and "tcgen05_tf32_pair" in wide["peak_source"]
    assert abs(wide["frac"] - wide["achieved"] / wide["peak"]) < 1e-3
    assert abs(wide["step_achieved"] - flop / step_ms / 1e9) < 0.01
    assert wide["traffic"] == 695.2e6 and wide["bound"] == "tensor" and wide["unit"] == "TFLOP/s"
    assert abs(wide["cublas_derived"]["peak"] - 1679.7 / 6) < 0.01
    assert wide["nominal"]["peak"] == round(1100 / 3, 1) and 0 < wide["nominal"]["frac"] < 1
    assert wide["algorithmic_bytes"] == 5 * 4096 * 4096 * 4
    fallback = bench._roofline("tc", 256, True, 2, gemm_ms, step_ms, peaks, "measured", None)
    assert abs(fallback["peak"] - 1679.7 / 6) < 0.01 and "bf16 burst" in fallback["peak_source"]
    narrow = bench._roofline("tc", 128, True, 1, 0.577, 0.658, peaks, "measured", ceil)
    assert narrow["kernel"].endswith("256x128 tiles on CTA pairs)")
    assert narrow["traffic"] == 923.4e6
    single = bench._roofline("tc", 128, False, 1, 0.6, 0.7, peaks, "measured", ceil)
    assert single["traffic"] is None and abs(single["peak"] - 1112.6 / 3) < 0.01
    ffma = bench._roofline("simt", 0, False, 1, 3.7, 3.7, peaks, "measured", ceil)
    assert ffma["kernel"] == "FFMA SIMT SGEMM" and "nominal" not in ffma
    assert ffma["peak"] == 71.7
    ffma_nom = bench._roofline("simt", 0, False, 1, 3.7, 3.7, peaks, "measured", None)
    assert abs(ffma_nom["peak"] - 148 * 128 * 2 * 1.965e-3) < 0.01
    json.dumps(wide)


def test_fused_replication_roofline():
    """The sharded secondary's roofline of the fused GEMM + P2P replication:
    the slower of the rank's FLOPs at the bf16 burst rate and its NVLink bytes
    at the measured peer-copy rate, against the measured time."""
    sys.path.insert(0, ROOT)
    import bench
    # cfg5 on 4 GPUs: 64 GEMMs of 2048^3 per rank, 1.5 GiB sent per rank
    r = {"with_p2p_epilogue": {"ms": 2.56}}
    bench._fused_roofline(r, 64 * 2.0 * 2048 ** 3, 3 * 64 * 2048 * 2048 * 2, 1684.4)
    rf = r["p2p_roofline"]
    assert rf["bound"] == "nvlink"
    assert abs(rf["link_ms"] - 3 * 64 * 2048 * 2048 * 2 / 770e9 * 1e3) < 1e-3
    assert abs(rf["math_ms"] - 64 * 2.0 * 2048 ** 3 / 1684.4e12 * 1e3) < 1e-3
    assert rf["target_ms"] == rf["link_ms"] and abs(rf["frac"] - rf["target_ms"] / 2.56) < 1e-3
    # 16384^3 column shard on 2 GPUs: tensor-bound
    r = {"with_p2p_epilogue": {"ms": 3.3}}
    bench._fused_roofline(r, 2.0 * 16384 * 8192 * 16384, 8192 * 16384 * 2, 1684.4)
    assert r["p2p_roofline"]["bound"] == "tensor"
    assert 0 < r["p2p_roofline"]["frac"] <= 1
