"""bench.py's pieces that need no GPU: the published-number table, the flop counts, the
reference arm's line (same config and step count as the GPU arm's), and that no committed
text file is read to produce a figure.
"""

import json
import re
import subprocess
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402
import rlenv_flops  # noqa: E402


def test_published_numbers_match_their_keys():
    value, source = bench.published("acrobot_step", 262_144)
    assert value == pytest.approx(1.123e9, rel=0.01) and "M3 Pro" in source
    assert bench.published("acrobot_step", 1)[0] is None


def test_legged_flop_counts_follow_the_kernel():
    ours = rlenv_flops.legged_flops(4, 8)["flops"]
    dense = rlenv_flops.legged_reference_flops(4, 8)["flops"]
    assert dense == 16417 and ours < dense
    assert rlenv_flops.legged_flops(4, 16)["flops"] > ours > rlenv_flops.legged_flops(4, 4)["flops"]
    assert rlenv_flops.legged_flops(1, 1)["flops"] < rlenv_flops.legged_flops(2, 8)["flops"] < ours


def test_bench_reads_no_committed_text_for_its_figures():
    """The only file bench.py reads a figure from is the driver-written MEASURED_PEAKS.json; the
    ncu summaries under profiles/ are cross-checks and are never parsed."""
    src = (ROOT / "bench.py").read_text()
    paths = set(re.findall(r'/ "([^"]+)"', src))
    assert paths <= {"MEASURED_PEAKS.json", "metal-rl-envs_b200", "baseline", "_ref", "acrobot_np.py"}, paths
    assert "profiles" not in src.replace("profiles/ (not read here)", "")


def test_reference_arm_prints_the_gpu_arms_config_and_steps_without_a_gpu():
    """--impl reference runs the reference's numpy step (or its restatement) on host cores."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "3",
                          "--warmup", "1", "--n", "4096", "--t", "2", "--cpu-seconds", "2"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["steps"] == 3 and line["warmup"] == 1
    assert line["config"] == bench.default_config(4096, 2, 1)
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
