"""rlenv_es_centered_ranks_static, the rank entry point that allocates nothing (its scratch is a
fixed array inside the library), against rlenv_es_centered_ranks_sorted with caller scratch.
Two calls in a row reuse the array with the first call's keys still in it. This file is
collected last, so it runs both alone and after every other test."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import es as oes
from parity import to_np

MAX_MEMBERS = 65_536


def _with_caller_scratch(rl, fit):
    p = fit.shape[0]
    out = torch.empty_like(fit)
    need = rl.lib().es_ranks_scratch_bytes(p)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=fit.device)
    rl.check(rl.lib().es_centered_ranks_sorted(fit.data_ptr(), p, out.data_ptr(), scratch.data_ptr(), need,
                                               rl.stream_ptr(fit.device)))
    return to_np(out)


def _with_static_scratch(rl, fit):
    out = torch.empty_like(fit)
    rl.check(rl.lib().es_centered_ranks_static(fit.data_ptr(), fit.shape[0], out.data_ptr(),
                                               rl.stream_ptr(fit.device)))
    return to_np(out)


def test_oversize_and_bad_arguments_are_rejected_without_a_launch():
    import rlenv_lib as rl

    lib = rl.load()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: each call is rejected first
    assert lib.es_centered_ranks_static(fake, MAX_MEMBERS + 1, fake, None) == -1
    assert lib.es_centered_ranks_static(fake, 1, fake, None) == -1
    assert lib.es_centered_ranks_static(None, 100, fake, None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("p", [3, 4096, 5000, MAX_MEMBERS])
def test_static_scratch_equals_caller_scratch_on_two_calls_in_a_row(cuda, p):
    import rlenv_lib as rl

    r = np.random.default_rng(p)
    first = torch.from_numpy(r.normal(size=p).astype(np.float32)).to(cuda)
    second = torch.from_numpy(r.integers(0, max(2, p // 16), p).astype(np.float32)).to(cuda)  # ties
    got1 = _with_static_scratch(rl, first)
    got2 = _with_static_scratch(rl, second)
    np.testing.assert_array_equal(got1, _with_caller_scratch(rl, first))
    np.testing.assert_array_equal(got2, _with_caller_scratch(rl, second))
    # and the reference's centred ranks (es.py:214-215), ties broken by member index
    np.testing.assert_allclose(got2, oes.centered_ranks(to_np(second)), rtol=0, atol=1e-7)


@pytest.mark.gpu
def test_a_warm_call_allocates_no_device_memory(cuda):
    """The point of the entry point: once its first call on the device has set up, a call at the
    largest size leaves the device's free memory exactly where it was."""
    import rlenv_lib as rl

    fit = torch.from_numpy(np.random.default_rng(7).normal(size=MAX_MEMBERS).astype(np.float32)).to(cuda)
    out = torch.empty_like(fit)
    sp = rl.stream_ptr(cuda)
    rl.check(rl.lib().es_centered_ranks_static(fit.data_ptr(), MAX_MEMBERS, out.data_ptr(), sp))
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info(cuda)[0]
    rl.check(rl.lib().es_centered_ranks_static(fit.data_ptr(), MAX_MEMBERS, out.data_ptr(), sp))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda)[0] == before
