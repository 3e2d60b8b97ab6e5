"""bench.py's host-side contract, without a GPU: the tensor-peak choice by
the length of the timed region, the gradient-update description, and the
reference arm's JSON line (the reference's CPU algorithm, run here)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_tensor_peak_is_chosen_by_the_timed_region():
    peaks = {"bf16_tflops": 1661.6, "bf16_tflops_sustained": 1412.9, "source": "MEASURED_PEAKS.json"}
    p, src = bench._tensor_peak(peaks, 0.11)
    assert p == 1661.6 and "burst" in src
    p, src = bench._tensor_peak(peaks, bench.SUSTAINED_AFTER_S)
    assert p == 1412.9 and "sustained" in src
    p, _ = bench._tensor_peak({"bf16_tflops": 1590.0, "source": "fallback"}, 30.0)
    assert p == 1590.0  # no sustained figure: the burst one


def test_update_path_names_the_collective():
    from jax4j_b200 import psum_sgd
    assert "no collective" in bench.update_path(1)
    was = psum_sgd.ENABLED
    try:
        psum_sgd.ENABLED = False
        assert "NCCL" in bench.update_path(8)
        psum_sgd.ENABLED = True
        assert "peer memory" in bench.update_path(8)
    finally:
        psum_sgd.ENABLED = was


def test_reference_arm_prints_one_line_with_its_baseline():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "samples/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=120, cwd=ROOT, env=env)
    assert r.returncode == 0 and not r.stdout.strip()
