"""bench.py helpers that need no GPU: the roofline's algorithmic bytes (the per-unit
figures of the workload), the DRAM traffic recorded in the committed ncu summaries, the
peak, and the reference arm's JSON line (a short CPU run of the C oracle)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_algorithmic_bytes_of_the_headline_shapes():
    # packed int4 weights + fp32 scales (per-row: one per row; group-128: one per 128 columns)
    assert bench.algorithmic_bytes(262144, 2048, 128) == 268435456 + 16777216
    assert bench.algorithmic_bytes(262144, 2048, 0) == 268435456 + 1048576
    assert bench.algorithmic_bytes(262144, 2048, 128, scale_bytes=2) == 268435456 + 8388608
    assert bench.algorithmic_bytes(128256, 2048, 128) == 131334144 + 8208384


def test_ncu_traffic_from_committed_profiles():
    g128 = bench.ncu_traffic("k_gemv_tma_g128_262144x2048.md")
    row = bench.ncu_traffic("k_gemv_tma_row_262144x2048.md")
    assert isinstance(g128, int) and isinstance(row, int)
    # traffic per launch within 3% of the algorithmic bytes: no re-reads (the excess is the
    # output and counter writes, 4-7 MB per launch in the captures)
    assert abs(g128 / bench.algorithmic_bytes(262144, 2048, 128) - 1) < 0.03
    assert abs(row / bench.algorithmic_bytes(262144, 2048, 0) - 1) < 0.03
    assert bench.ncu_traffic("no_such_profile.md") is None


def test_peak_is_the_measured_copy_bandwidth():
    peak, src = bench.load_peaks()
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            assert peak == float(json.load(f)["hbm_gbs"]) and src.startswith("measured")
    else:
        assert peak == 6650.0 and "fallback" in src


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "µs"
    assert line["higher_is_better"] is False and line["value"] > 0
    assert line["config"]["workload"] == "g128 int4 GEMV 262144x2048, batch 1"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # the full matrix every step (no extrapolation), and the reference's torch expression beside it
    assert "full 262144x2048" in line["cpu_baseline"]["sample"] and "median" in line["cpu_baseline"]["sample"]
    assert "same_inputs_as_gpu_arm" in line["config"]
    assert line["reference_torch"]["value"] > 0 and "repeat_interleave" in line["reference_torch"]["expr"]


def test_llama8b_shapes_shard_evenly_over_1_to_8_gpus():
    from w4a16.tp import shard_bounds

    for _, rows, cols in bench.LLAMA8B_SHAPES:
        assert cols % 256 == 0                        # the TMA path of the kernel
        for world in (1, 2, 4, 8):
            spans = [shard_bounds(rows, world, r) for r in range(world)]
            assert len({hi - lo for lo, hi in spans}) == 1, (rows, world)  # equal shards
            assert (spans[0][1] - spans[0][0]) % 16 == 0
