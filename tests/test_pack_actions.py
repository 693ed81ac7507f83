"""The packed action format (RLENV_U2) on the host: rlenv_lib.pack_actions packs (T, N)
actions along time, byte (r, i) holding environment i's steps 4r .. 4r + 3 in two bits each,
and the step calls check PackedActions against the batch."""

import numpy as np
import pytest
import torch

import rlenv_lib


def _pack_loop(a):
    a = np.asarray(a)
    if a.ndim == 1:
        a = a[None]
    T, n = a.shape
    out = np.zeros(((T + 3) // 4, n), np.uint8)
    for t in range(T):
        for i in range(n):
            out[t // 4, i] |= (int(a[t, i]) & 3) << (2 * (t % 4))
    return out


@pytest.mark.parametrize("shape", [(1,), (5,), (1, 3), (3, 7), (4, 9), (5, 2), (13, 64), (1000, 3)])
def test_pack_actions_layout(shape):
    a = np.random.default_rng(sum(shape)).integers(0, 3, shape)
    got = rlenv_lib.pack_actions(torch.from_numpy(a))
    T = shape[0] if len(shape) == 2 else 1
    n = shape[-1]
    assert got.steps == T and got.bits.dtype == torch.uint8 and tuple(got.bits.shape) == ((T + 3) // 4, n)
    assert np.array_equal(got.bits.numpy(), _pack_loop(a))
    # every step's action comes back out, and the steps past T are zero
    bits = got.bits.numpy()
    back = np.stack([(bits >> (2 * u)) & 3 for u in range(4)], 1).reshape(-1, n)
    assert np.array_equal(back[:T], a.reshape(T, n)) and not back[T:].any()


def test_pack_actions_takes_numpy_and_every_integer_dtype():
    a = np.array([[0, 1, 2, 1, 0], [2, 2, 0, 1, 1]])
    want = _pack_loop(a)
    for t in (np.int64, np.int32, np.uint8):
        assert np.array_equal(rlenv_lib.pack_actions(a.astype(t)).bits.numpy(), want)
    with pytest.raises(ValueError):
        rlenv_lib.pack_actions(a.astype(np.float32))


def test_packed_actions_are_checked_against_the_batch():
    dev = torch.device("cpu")
    ok = rlenv_lib.PackedActions(torch.zeros((2, 5), dtype=torch.uint8), 7).checked(5, dev)
    assert ok.shape == (2, 5)
    with pytest.raises(ValueError):
        rlenv_lib.PackedActions(torch.zeros((2, 5), dtype=torch.int32), 7).checked(5, dev)   # not bytes
    with pytest.raises(ValueError):
        rlenv_lib.PackedActions(torch.zeros((7, 5), dtype=torch.uint8), 7).checked(5, dev)   # unpacked rows
    with pytest.raises(ValueError):
        rlenv_lib.PackedActions(torch.zeros((2, 4), dtype=torch.uint8), 7).checked(5, dev)   # other batch
