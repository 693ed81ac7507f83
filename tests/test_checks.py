"""The check build (librlenv_checks.so, -DRLENV_CHECKS): kernels record an action outside its
body's range and a non-finite output in a device word, which rlenv_checks_status reads and
clears; they never trap. It stands in for compute-sanitizer, which is closed on this pool.

The CPU tests load both libraries (no GPU call reaches a device): the normal build answers
"unsupported", and the check build's reporting path turns a failed device read into a CUDA
error code instead of a crash. The GPU tests run small ragged batches through the check build:
clean inputs leave the word at zero, an out-of-range action and a NaN state set their bits."""

import ctypes

import numpy as np
import pytest

from conftest import PKG

RLENV_EUNSUPPORTED = -2


def _load(name):
    import rlenv_lib

    lib = ctypes.CDLL(str(PKG / name))
    for fn, args in rlenv_lib._SIGNATURES.items():
        getattr(lib, fn).argtypes = args
        getattr(lib, fn).restype = rlenv_lib._RESTYPES.get(fn, ctypes.c_int)
    return lib


def _status(lib, clear=1):
    word = ctypes.c_uint(0xDEAD)
    rc = lib.rlenv_checks_status(ctypes.byref(word), clear)
    return rc, word.value


def test_normal_build_reports_unsupported_without_a_gpu():
    rc, word = _status(_load("librlenv.so"))
    assert rc == RLENV_EUNSUPPORTED and word == 0


def test_check_build_reporting_path_fails_cleanly_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("this is the no-device path")
    lib = _load("librlenv_checks.so")
    rc, word = _status(lib)
    assert rc > 0 and word == 0  # a CUDA error code (no device), not a crash
    assert lib.rlenv_checks_status(None, 1) == -1


@pytest.mark.gpu
def test_check_build_flags_bad_actions_and_non_finite_outputs(cuda):
    import torch

    lib = _load("librlenv_checks.so")
    sp = torch.cuda.current_stream(cuda).cuda_stream
    assert _status(lib)[0] == 0  # clears anything earlier
    for n in (1, 33, 257):
        r = np.random.default_rng(n)
        st = torch.from_numpy(r.uniform(-0.05, 0.05, (4, n)).astype(np.float32)).to(cuda)
        out = torch.empty_like(st)
        rew = torch.empty(n, device=cuda)
        dn = torch.empty(n, dtype=torch.uint8, device=cuda)

        def step(fn, state, action):
            a = torch.from_numpy(np.asarray(action, np.int32)).to(cuda)
            assert fn(state.data_ptr(), a.data_ptr(), 0, 3, n, 0, out.data_ptr(), rew.data_ptr(), dn.data_ptr(), sp) == 0
            torch.cuda.synchronize()
            return _status(lib)

        ok = r.integers(0, 2, n)
        assert step(lib.rlenv_cartpole_step, st, ok) == (0, 0)
        assert step(lib.rlenv_acrobot_step, st, ok) == (0, 0)
        bad = ok.copy()
        bad[n // 2] = 7
        assert step(lib.rlenv_acrobot_step, st, bad) == (0, 1)
        assert _status(lib) == (0, 0), "read with clear zeroes the word"
        nan = st.clone()
        nan[1, n - 1] = float("nan")
        assert step(lib.rlenv_cartpole_step, nan, ok) == (0, 2)
        # the pendulum (registers and the long-chain shared-memory form) and the legged body
        for k in (4, 20):
            ps = torch.from_numpy(r.uniform(-0.1, 0.1, (2 * k, n)).astype(np.float32)).to(cuda)
            po = torch.empty_like(ps)
            a = torch.from_numpy(r.integers(0, 3, n).astype(np.int32)).to(cuda)
            assert lib.rlenv_pendulum_aba_step(k, ps.data_ptr(), a.data_ptr(), 0, 3, n, 0, po.data_ptr(),
                                               rew.data_ptr(), dn.data_ptr(), sp) == 0
            torch.cuda.synchronize()
            assert _status(lib) == (0, 0), k
        ls = torch.from_numpy((np.array([0, 1, 0, -0.25, 0.25] + [0] * 5, np.float32)[:, None]
                               + r.uniform(-0.05, 0.05, (10, n))).astype(np.float32)).to(cuda)
        stand = torch.from_numpy(np.array([0, 1, 0, -0.25, 0.25] + [0] * 5, np.float32)).to(cuda)
        lo = torch.empty_like(ls)
        la = torch.from_numpy(r.integers(0, 9, n).astype(np.int32)).to(cuda)
        assert lib.rlenv_legged_step(2, 8, ls.data_ptr(), la.data_ptr(), 0, 3, stand.data_ptr(), 0.0, None, n, 0,
                                     lo.data_ptr(), rew.data_ptr(), dn.data_ptr(), None, sp) == 0
        torch.cuda.synchronize()
        assert _status(lib) == (0, 0)
        la[0] = 9  # 3^2 actions for two legs
        assert lib.rlenv_legged_step(2, 8, ls.data_ptr(), la.data_ptr(), 0, 3, stand.data_ptr(), 0.0, None, n, 0,
                                     lo.data_ptr(), rew.data_ptr(), dn.data_ptr(), None, sp) == 0
        torch.cuda.synchronize()
        assert _status(lib) == (0, 1)


@pytest.mark.gpu
def test_check_build_flags_in_the_tensor_memory_kernel(cuda):
    """K = 64 on a batch that fills the GPU runs the long-chain pendulum's mixed kernel (four
    tensor-memory warps per block beside shared-memory ones): a clean batch leaves the word at
    zero, a bad action in a tensor-memory warp (the first environment) and one in a
    shared-memory warp (the 200th) set bit 1, and a non-finite state sets bit 2."""
    import torch

    lib = _load("librlenv_checks.so")
    sp = torch.cuda.current_stream(cuda).cuda_stream
    assert _status(lib)[0] == 0
    k = 64
    n = 32 * torch.cuda.get_device_properties(0).multi_processor_count * 7
    r = np.random.default_rng(64)
    ps = torch.from_numpy(r.uniform(-0.1, 0.1, (2 * k, n)).astype(np.float32)).to(cuda)
    po = torch.empty_like(ps)
    rew = torch.empty(n, device=cuda)
    dn = torch.empty(n, dtype=torch.uint8, device=cuda)

    def step(state, action):
        a = torch.from_numpy(np.asarray(action, np.int32)).to(cuda)
        assert lib.rlenv_pendulum_aba_step(k, state.data_ptr(), a.data_ptr(), 0, 3, n, 0, po.data_ptr(),
                                           rew.data_ptr(), dn.data_ptr(), sp) == 0
        torch.cuda.synchronize()
        return _status(lib)

    ok = r.integers(0, 3, n)
    assert step(ps, ok) == (0, 0)
    for where in (0, 200):
        bad = ok.copy()
        bad[where] = 5
        assert step(ps, bad) == (0, 1), where
    nan = ps.clone()
    nan[3, 7] = float("nan")
    assert step(nan, ok)[1] & 2


@pytest.mark.gpu
def test_check_build_flags_packed_actions_and_the_one_warp_pendulum(cuda):
    """Packed actions (RLENV_U2) can hold 3, outside both classic bodies' ranges: the T-step
    kernels flag it on the step that reads it, at one and at four environments per thread
    (CartPole from N = 4 x 32 x 32 x SMs). The one-warp articulated body (every K above 64)
    flags a bad action and a non-finite state as the other forms do."""
    import torch

    import rlenv_lib

    lib = _load("librlenv_checks.so")
    sp = torch.cuda.current_stream(cuda).cuda_stream
    assert _status(lib)[0] == 0
    r = np.random.default_rng(3)
    for n in (33, 4 * 32 * 32 * torch.cuda.get_device_properties(0).multi_processor_count):
        st = torch.from_numpy(r.uniform(-0.05, 0.05, (4, n)).astype(np.float32)).to(cuda)
        out = torch.empty_like(st)
        T = 6
        acts = torch.from_numpy(r.integers(0, 2, (T, n))).to(cuda)
        for fn in (lib.rlenv_cartpole_step_many, lib.rlenv_acrobot_step_many):
            for bad in (False, True):
                a = acts.clone()
                if bad:
                    a[5, n - 1] = 3
                bits = rlenv_lib.pack_actions(a).bits
                assert fn(st.data_ptr(), bits.data_ptr(), rlenv_lib.U2, 1, T, n, 0, out.data_ptr(), None, None, None,
                          None, sp) == 0
                torch.cuda.synchronize()
                assert _status(lib) == (0, 1 if bad else 0), (n, bad)
    k, n = 100, 40
    ps = torch.from_numpy(r.uniform(-0.1, 0.1, (2 * k, n)).astype(np.float32)).to(cuda)
    po = torch.empty_like(ps)
    rew = torch.empty(n, device=cuda)
    dn = torch.empty(n, dtype=torch.uint8, device=cuda)

    def step(state, action):
        a = torch.from_numpy(np.asarray(action, np.int32)).to(cuda)
        assert lib.rlenv_pendulum_aba_step(k, state.data_ptr(), a.data_ptr(), 0, 3, n, 0, po.data_ptr(),
                                           rew.data_ptr(), dn.data_ptr(), sp) == 0
        torch.cuda.synchronize()
        return _status(lib)

    ok = r.integers(0, 3, n)
    assert step(ps, ok) == (0, 0)
    bad = ok.copy()
    bad[n - 1] = 4
    assert step(ps, bad) == (0, 1)
    nan = ps.clone()
    nan[k + 50, 3] = float("nan")
    assert step(nan, ok) == (0, 2)
