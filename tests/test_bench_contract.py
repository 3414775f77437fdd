"""bench.py's reference arm (the CPU oracle port timed on the host cores) runs
without a GPU and prints one JSON line with the keys the benchmark contract
asks for. Config 0 keeps it to a few seconds."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--config", "0",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [s for s in r.stdout.splitlines() if s.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]


def test_byte_models_and_rooflines():
    """The per-kernel byte models add up to the step's algorithmic bytes and
    the rooflines are computed from stage times and the raster counters."""
    sys.path.insert(0, REPO)
    import bench
    m = bench.byte_models(n=3_000_000, n_vis=2_670_000, K=15, T=63_860, P=4946 * 3286, emitted=25_000_000,
                          kept=22_900_000)
    # SH3: 232 B of parameters per Gaussian; the fused VJP + Adam moves
    # 6 x 232 + 92 B per Gaussian
    assert bench.param_bytes(15) == 232
    assert m["project_backward_adam"] == 3_000_000 * (6 * 232 + 92)
    assert m["loss_ssim"] == 36 * 4946 * 3286
    ra = bench.roofline_all({"loss_ssim": 1.0, "rasterize_backward": 5.0}, m, 6545.0)
    assert set(ra) == {"loss_ssim", "rasterize_backward"}
    assert abs(ra["loss_ssim"]["gb_s"] - m["loss_ssim"] / 1e-3 / 1e9) < 0.1
    cr = bench.compute_roofline({"rasterize_forward": 4.0, "rasterize_backward": 5.0},
                                [300_000_000, 40_000_000, 25_000_000, 310_000_000], 1965.0)
    assert cr["peak"] == 148 * 4 * 1965e6
    b = cr["rasterize_backward"]
    assert b["visits"] == 25_000_000 and abs(b["pair_evals_per_s"] - 32 * 25e6 / 5e-3) < 1
    assert 0 < b["useful_lane_frac"] <= 1
