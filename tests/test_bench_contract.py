"""bench.py's pieces that need no GPU: the figures it reads from the committed ncu summary,
the instruction-issue view built from them, the flop counts and the published-number table.
"""

import json
import subprocess
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402
import rlenv_flops  # noqa: E402


def test_profile_figures_are_present_and_plausible():
    traffic = bench.profiled("traffic_bytes_per_launch")
    inst = bench.profiled("inst_per_env_step")
    algorithmic = rlenv_flops.step_many_bytes(4, 262_144, 1_000, 1, True)
    assert traffic is not None and 0.9 * algorithmic <= traffic <= 1.1 * algorithmic
    # at least one instruction per algorithmic flop's FMA pair, fewer than the old sincosf build
    assert inst is not None and rlenv_flops.ACROBOT["flops"] / 2 <= inst <= 500


def test_issue_view_is_a_fraction_of_the_scheduler_limit():
    view = bench.issue_view(50e9, 1965.0, 148)
    inst = bench.profiled("inst_per_env_step")
    assert view["peak"] == pytest.approx(148 * 4 * 32 * 1965.0e6 / 1e9)
    assert view["achieved"] == pytest.approx(50e9 * inst / 1e9)
    assert 0 < view["frac"] < 1
    assert bench.issue_view(50e9, None, 148) is None


def test_published_numbers_match_their_keys():
    value, source = bench.published("acrobot_step", 262_144)
    assert value == pytest.approx(1.123e9, rel=0.01) and "M3 Pro" in source
    assert bench.published("acrobot_step", 1)[0] is None


def test_legged_flop_counts_follow_the_kernel():
    closed = rlenv_flops.legged_flops(4, 8)["flops"]
    dense = rlenv_flops.legged_reference_flops(4, 8)["flops"]
    assert closed == 8812 and dense == 16417
    assert rlenv_flops.legged_flops(4, 16)["flops"] > closed > rlenv_flops.legged_flops(4, 4)["flops"]


def test_reference_arm_prints_unavailable_or_a_line_without_a_gpu():
    """--impl reference runs the oracle port on host cores; it needs no GPU."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--n", "4096", "--t", "2"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
