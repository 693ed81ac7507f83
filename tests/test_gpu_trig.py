"""The kernels' sine and cosine (sincos_fast, csrc/common.cuh) on the device.

Every physics kernel takes its trigonometry from sincos_fast. This checks its error against
float64 sin and cos, in float32 ulps of the exact value, next to CUDA's sincosf and float32
numpy on the same inputs. The probe is compiled here from tests/trig_probe.cu.
"""

import ctypes
import subprocess

import numpy as np
import pytest
import torch

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu

ULP_BOUND = 1.6  # both results, |x| <= 1024


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    import rlenv_build

    so = tmp_path_factory.mktemp("trig") / "trig_probe.so"
    cmd = [rlenv_build.nvcc(), *rlenv_build.ARCH, "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-shared", "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}", f"-I{PKG / 'csrc'}",
           str(ROOT / "tests" / "trig_probe.cu"), "-o", str(so)]
    subprocess.run(cmd, check=True, capture_output=True)
    lib = ctypes.CDLL(str(so))
    lib.trig_probe.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64]
    lib.sfu_probe.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64]
    lib.near_probe.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64]

    def run(x, sfu=False, near=False):
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        outs = [torch.empty_like(xd) for _ in range(2 if (sfu or near) else 4)]
        entry = lib.near_probe if near else lib.sfu_probe if sfu else lib.trig_probe
        assert entry(xd.data_ptr(), *(o.data_ptr() for o in outs), xd.numel()) == 0
        return [o.cpu().numpy() for o in outs]

    return run


def _ulps(got, exact):
    spacing = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
    return np.abs(got.astype(np.float64) - exact) / spacing


def _inputs(limit, seed=0):
    r = np.random.default_rng(seed)
    near_quadrants = np.arange(-int(limit / (np.pi / 2)), int(limit / (np.pi / 2)) + 1) * (np.pi / 2)
    near = (near_quadrants[:, None] + np.linspace(-1e-5, 1e-5, 41)[None, :]).ravel()
    x = np.concatenate([r.uniform(-limit, limit, 4_000_000), np.linspace(-limit, limit, 1_000_001), near])
    x = x.astype(np.float32)
    return x[np.abs(x) <= limit]


@pytest.mark.parametrize("limit", [np.pi, 40.0, 1024.0])
def test_sincos_fast_error_in_ulps(probe, limit):
    x = _inputs(limit)
    s, c, s_lib, c_lib = probe(x)
    xs = x.astype(np.float64)
    es, ec = _ulps(s, np.sin(xs)), _ulps(c, np.cos(xs))
    lib_s, lib_c = _ulps(s_lib, np.sin(xs)), _ulps(c_lib, np.cos(xs))
    np_s, np_c = _ulps(np.sin(x), np.sin(xs)), _ulps(np.cos(x), np.cos(xs))
    print(f"|x| <= {limit}: sin {es.max():.3f} cos {ec.max():.3f} ulp; sincosf {lib_s.max():.3f} "
          f"{lib_c.max():.3f}; numpy float32 {np_s.max():.3f} {np_c.max():.3f}")
    assert es.max() <= ULP_BOUND and ec.max() <= ULP_BOUND


def test_sincos_fast_outside_the_fast_range_is_sincosf(probe):
    x = np.array([1024.5, -2000.0, 1e5, -3e7, 1e30, np.inf, -np.inf, np.nan], np.float32)
    s, c, s_lib, c_lib = probe(x)
    np.testing.assert_array_equal(s, s_lib)
    np.testing.assert_array_equal(c, c_lib)
    assert np.isnan(s[-3:]).all() and np.isnan(c[-3:]).all()


def test_sincos_fast_branch_placements_agree(probe):
    """The out-of-line (kShared) and inline (kInline) placements of sincosf's branch give the
    same bits on both sides of 1,024 rad (the probe turns a mismatch into NaN)."""
    r = np.random.default_rng(1)
    x = np.concatenate([r.uniform(-2048, 2048, 1_000_000), r.uniform(-1e6, 1e6, 10_000)]).astype(np.float32)
    s, _, _, _ = probe(x)
    assert not np.isnan(s).any()


def test_sincos_fast_exact_points(probe):
    x = np.array([0.0, 1e-30, -1e-30, 1e-7], np.float32)
    s, c, _, _ = probe(x)
    np.testing.assert_array_equal(s[1:], x[1:])  # sin x = x below half an ulp of x^3/6
    np.testing.assert_array_equal(c, np.ones(4, np.float32))
    assert s[0] == 0.0


# CUDA documents __sinf and __cosf within 2^-21.41 (3.6e-7) absolute on [-pi, pi]. The
# reduced argument carries its own rounding and, where the quotient rounds the other way,
# lies just past pi. Measured over these inputs on a B200: 5.9e-7 at worst.
SFU_ABS_BOUND = 8e-7


def test_sincos_sfu_absolute_error(probe):
    """sincos_sfu (the legged bodies' and the ES rollouts' leg trig): within the special function
    unit's bound over the range the bodies use, and far beyond it."""
    x = _inputs(1024.0, seed=2)
    s, c = probe(x, sfu=True)
    xs = x.astype(np.float64)
    es, ec = np.abs(s - np.sin(xs)).max(), np.abs(c - np.cos(xs)).max()
    print(f"sincos_sfu |x| <= 1024: sin {es:.3g} cos {ec:.3g} absolute (bound {SFU_ABS_BOUND:.3g})")
    assert es <= SFU_ABS_BOUND and ec <= SFU_ABS_BOUND


# sincos_sfu_near (the Acrobot's and the long-chain pendulum's trig) has no reduction in front:
# the unit's own error grows with |x|. Measured over every float32 in each range on a B200:
# 4.04e-7, 6.5e-7, 1.21e-6 and 2.27e-6; the bounds keep a margin.
NEAR_ABS_BOUNDS = [(np.pi, 5e-7), (4.0, 8e-7), (8.0, 1.4e-6), (16.0, 2.6e-6)]


@pytest.mark.parametrize("limit,bound", NEAR_ABS_BOUNDS)
def test_sincos_sfu_near_absolute_error(probe, limit, bound):
    """The unreduced unit within its measured bound on each range the kernels use it for: a
    wrapped angle (pi), the Acrobot's stage angles and the pendulum's joint angles (8)."""
    x = _inputs(limit, seed=3)
    s, c = probe(x, near=True)
    xs = x.astype(np.float64)
    es, ec = np.abs(s - np.sin(xs)).max(), np.abs(c - np.cos(xs)).max()
    print(f"sincos_sfu_near |x| <= {limit:.4g}: sin {es:.3g} cos {ec:.3g} absolute (bound {bound:.3g})")
    assert es <= bound and ec <= bound


def test_sincos_sfu_near_equals_sincos_sfu_within_pi(probe):
    """For |x| <= float(pi) the reduction's quotient is zero, so both forms give the same bits
    (zero aside: the reduction turns -0 into +0)."""
    r = np.random.default_rng(4)
    x = np.concatenate([r.uniform(-np.pi, np.pi, 2_000_000), np.linspace(-np.pi, np.pi, 100_001)]).astype(np.float32)
    x = x[(np.abs(x) <= np.float32(np.pi)) & (x != 0)]
    s1, c1 = probe(x, sfu=True)
    s2, c2 = probe(x, near=True)
    np.testing.assert_array_equal(s1.view(np.uint32), s2.view(np.uint32))
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))
