"""The C ABI library builds, loads and exports every entry point include/rlenv.h declares, and
rejects bad arguments with a status code before launching anything (CPU; no kernel runs)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from conftest import PKG, ROOT

HEADER = ROOT / "include" / "rlenv.h"


def _declared():
    return sorted(set(re.findall(r"RLENV_API\s+(?:int64_t|int|const char\*)\s+(rlenv_\w+)\(", HEADER.read_text())))


@pytest.fixture(scope="module")
def lib():
    import rlenv_build
    import rlenv_lib

    rlenv_build.build()
    return rlenv_lib.load()


def test_header_and_binding_agree():
    import rlenv_lib

    assert _declared() == rlenv_lib.exported_symbols()


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(PKG / "librlenv.so")], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (rlenv_\w+)", out))
    assert set(_declared()) <= exported, set(_declared()) - exported
    for name in _declared():
        assert getattr(lib.cdll, name) is not None


def test_version_and_messages(lib):
    assert lib.abi_version() == 2
    assert "invalid" in lib.strerror(-1) and "instance" in lib.strerror(-2) and lib.strerror(0) == "ok"


def test_arguments_rejected_before_launch(lib):
    """Every one of these returns before any CUDA call, so it runs without a GPU."""
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: each call is rejected first
    assert lib.cartpole_step(fake, fake, 0, 1, -1, 0, fake, fake, fake, None) == -1   # negative n
    assert lib.cartpole_step(fake, fake, 7, 1, 4, 0, fake, fake, fake, None) == -1    # unknown dtype
    assert lib.cartpole_step(None, fake, 0, 1, 4, 0, fake, fake, fake, None) == -1    # null state
    assert lib.cartpole_step(None, None, 0, 1, 0, 0, None, None, None, None) == 0     # empty batch: nothing to do
    # packed actions (RLENV_U2 = 3) are for the CartPole and Acrobot kernels only
    assert lib.pendulum_aba_step(8, fake, fake, 3, 1, 4, 0, fake, fake, fake, None) == -1
    assert lib.pendulum_mm_step(4, 0, fake, fake, 3, 1, 4, 0, fake, fake, fake, None) == -1
    assert lib.legged_step(2, 8, fake, fake, 3, 1, fake, 0.0, None, 4, 0, fake, fake, fake, None, None) == -1
    assert lib.acrobot_step(None, None, 3, 1, 0, 0, None, None, None, None) == 0       # accepted there
    assert lib.pendulum_mm_step(17, 0, fake, fake, 0, 1, 4, 0, fake, fake, fake, None) == -2
    assert lib.pendulum_coop_step(3, fake, fake, 0, 1, 4, 0, fake, fake, fake, None) == -2
    assert lib.pendulum_aba_step(193, fake, fake, 0, 1, 4, 0, fake, fake, fake, None) == -2
    assert lib.legged_step(5, 8, fake, fake, 0, 1, fake, 0.0, None, 4, 0, fake, fake, fake, None, None) == -2
    assert lib.legged_step(2, 0, fake, fake, 0, 1, fake, 0.0, None, 4, 0, fake, fake, fake, None, None) == -1  # iters < 1
    assert lib.pendulum_mm_step_many(17, 0, fake, fake, 0, 1, 5, 4, 0, fake, None, None, None) == -2
    assert lib.pendulum_aba_step_many(8, fake, fake, 0, 1, -1, 4, 0, fake, None, None, None) == -1     # steps < 0
    assert lib.pendulum_coop_step_many(4, fake, None, 0, 1, 5, 4, 0, fake, None, None, None) == -1     # no actions
    assert lib.pendulum_aba_step_many(8, None, None, 0, 1, 0, 0, 0, None, None, None, None) == 0       # empty batch
    assert lib.legged_step_many(2, 8, fake, fake, 9, 1, fake, 0.0, None, 3, 4, 0, fake, None, None, None, None) == -1
    assert lib.hopper_step_many(1, fake, fake, 0, 1, fake, 3, -4, 0, fake, None, None, None) == -1     # n < 0
    assert lib.cartpole_rollout(fake, fake, 0, 4, 3, 10, fake, None) == -2                 # hidden 3 not built
    assert lib.legged_rollout(2, 16, 10, 8, 1.0, 0.0, 0.0, 0.0, fake, fake, 0, -1, fake, fake, None) == -1
    assert lib.es_centered_ranks(fake, 1, fake, None) == -1
    assert lib.es_ranks_scratch_bytes(4096) == 0 and lib.es_ranks_scratch_bytes(4097) == 16 * 4097
    assert lib.es_ranks_scratch_bytes(-1) == -1
    assert lib.es_centered_ranks_sorted(fake, 1, fake, None, 0, None) == -1                  # p < 2
    assert lib.es_centered_ranks_sorted(fake, 5000, fake, None, 0, None) == -1               # no scratch
    assert lib.es_centered_ranks_sorted(fake, 5000, fake, fake, 16 * 4999, None) == -1       # too little
    assert lib.es_centered_ranks_sorted(fake, 5000, fake, ctypes.c_void_p(0x1004), 16 * 5000, None) == -1  # misaligned
    assert lib.es_perturb(fake, 10, 0.1, 1, 1, 4, 6, 4, fake, None) == -1                   # past the population
    assert lib.es_update(fake, fake, 10, 4, 0.1, 0.0, 1, 1, fake, None) == -1               # sigma 0


def test_product_has_no_cpu_path():
    """The drop-in modules never import the oracle, and refuse to run without CUDA."""
    for f in PKG.glob("*.py"):
        text = f.read_text()
        assert "import oracle" not in text and "from oracle" not in text, f.name
    import rlenv_lib
    import torch

    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            rlenv_lib.device()


def test_a_c_host_compiles_links_and_calls_the_library(lib, tmp_path):
    """include/rlenv.h is plain C: a C99 program includes it, links librlenv.so and calls it."""
    exe = tmp_path / "c_abi_check"
    build = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                            str(ROOT / "tests" / "c_abi_check.c"), f"-L{PKG}", "-lrlenv", f"-Wl,-rpath,{PKG}",
                            "-o", str(exe)], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
