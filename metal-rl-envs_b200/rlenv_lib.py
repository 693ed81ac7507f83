"""ctypes binding of librlenv.so and the tensor plumbing shared by the drop-in modules.

The library's C ABI (include/rlenv.h) takes plain device pointers, sizes and a
cudaStream_t. This module turns torch tensors into those arguments and status
codes into Python exceptions:

- a negative status (a rejected argument, or parameters for which no kernel
  instance is built) raises ValueError, as the reference's
  `mx.fast.metal_kernel` raises on a template it cannot compile;
- a positive status is a CUDA error and raises RuntimeError.

There is no CPU path: a missing library or a missing CUDA device raises.
"""

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np
import torch

LIB_PATH = Path(__file__).resolve().parent / "librlenv.so"
# RLENV_LIBRARY=checks loads the check build instead (rlenv_build.build(checks=True))
CHECKS_LIB_PATH = Path(__file__).resolve().parent / "librlenv_checks.so"

I32, I64, U8, U2 = 0, 1, 2, 3
_DTYPES = {torch.int32: I32, torch.int64: I64, torch.uint8: U8, torch.bool: U8}

# name -> argument types; every function returns int except those in _RESTYPES
_RESTYPES = {"rlenv_es_ranks_scratch_bytes": c_int64}
_SIGNATURES = {
    "rlenv_abi_version": [],
    "rlenv_checks_status": [c_void_p, c_int],
    "rlenv_cartpole_step": [c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_cartpole_step_many": [c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_acrobot_step": [c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_acrobot_step_many": [c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_pendulum_mm_step": [c_int, c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_void_p, c_void_p,
                               c_void_p, c_void_p],
    "rlenv_pendulum_coop_step": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_void_p],
    "rlenv_pendulum_aba_step": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_void_p, c_void_p,
                                c_void_p, c_void_p],
    "rlenv_legged_step": [c_int, c_int, c_void_p, c_void_p, c_int, c_uint32, c_void_p, c_float, c_void_p, c_int64,
                          c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_hopper_step": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                          c_void_p, c_void_p],
    "rlenv_cartpole_rollout": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p],
    "rlenv_acrobot_rollout": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p],
    "rlenv_legged_rollout": [c_int, c_int, c_int, c_int, c_float, c_float, c_float, c_float, c_void_p, c_void_p,
                             c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "rlenv_legged_rollout_lanes": [c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_float, c_float, c_void_p,
                                   c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p],
    "rlenv_pendulum_mm_step_many": [c_int, c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64,
                                    c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_pendulum_coop_step_many": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64,
                                      c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_pendulum_aba_step_many": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64,
                                     c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_pendulum_aba_coop_step_many": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_int64, c_int64, c_int64,
                                          c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_legged_step_many": [c_int, c_int, c_void_p, c_void_p, c_int, c_uint32, c_void_p, c_float, c_void_p,
                               c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_hopper_step_many": [c_int, c_void_p, c_void_p, c_int, c_uint32, c_void_p, c_int64, c_int64, c_int64,
                               c_void_p, c_void_p, c_void_p, c_void_p],
    "rlenv_es_noise": [c_void_p, c_int64, c_int64, c_uint64, c_uint64, c_int64, c_void_p],
    "rlenv_es_perturb": [c_void_p, c_int64, c_float, c_uint64, c_uint64, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    "rlenv_es_centered_ranks": [c_void_p, c_int64, c_void_p, c_void_p],
    "rlenv_es_ranks_scratch_bytes": [c_int64],
    "rlenv_es_centered_ranks_sorted": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p],
    "rlenv_es_centered_ranks_static": [c_void_p, c_int64, c_void_p, c_void_p],
    "rlenv_es_update": [c_void_p, c_void_p, c_int64, c_int64, c_float, c_float, c_uint64, c_uint64, c_void_p, c_void_p],
    "rlenv_reset_uniform": [c_void_p, c_int, c_int64, c_void_p, c_float, c_uint32, c_int64, c_void_p],
}

_lib = None


class _Lib:
    """Attribute access to the library's entry points, loaded once."""

    def __init__(self, path):
        self.cdll = ctypes.CDLL(str(path))
        for name, args in _SIGNATURES.items():
            fn = getattr(self.cdll, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, c_int)
            setattr(self, name[len("rlenv_"):], fn)
        self.cdll.rlenv_strerror.argtypes = [c_int]
        self.cdll.rlenv_strerror.restype = ctypes.c_char_p

    def strerror(self, code):
        return self.cdll.rlenv_strerror(code).decode()


def load(path=None):
    """The loaded library. Raises if it has not been built (there is no fallback).
    RLENV_LIBRARY=checks in the environment selects the check build."""
    global _lib
    if path is None:
        path = CHECKS_LIB_PATH if os.environ.get("RLENV_LIBRARY") == "checks" else LIB_PATH
    if _lib is None:
        if not Path(path).exists():
            raise RuntimeError(f"{path} is not built; run metal-rl-envs_b200/rlenv_build.py "
                               "or __graft_entry__.build() first")
        _lib = _Lib(path)
    return _lib


def lib():
    return _lib if _lib is not None else load()


def exported_symbols():
    """Names of every entry point this binding declares (for ABI tests)."""
    return sorted(list(_SIGNATURES) + ["rlenv_strerror"])


CHECK_BITS = {1: "an action outside its body's range", 2: "a non-finite value written to an output"}


def checks_status(clear=True):
    """(word, [messages]) from the check build's device words (rlenv_checks_status), cleared
    with clear. Raises ValueError in the normal build, which records nothing."""
    word = ctypes.c_uint(0)
    check(lib().checks_status(ctypes.byref(word), 1 if clear else 0))
    return word.value, [m for b, m in CHECK_BITS.items() if word.value & b]


def check(rc):
    if rc == 0:
        return
    msg = lib().strerror(rc)
    if rc < 0:
        raise ValueError(f"librlenv rejected the call: {msg}")
    raise RuntimeError(f"CUDA error {rc} from librlenv: {msg}")


# ---- tensors -----------------------------------------------------------------------


def device():
    if not torch.cuda.is_available():
        raise RuntimeError("metal-rl-envs_b200 needs a CUDA device: there is no CPU path")
    return torch.device("cuda", torch.cuda.current_device())


def stream_ptr(dev=None):
    return torch.cuda.current_stream(dev).cuda_stream


def as_state(x, rows=None, name="state"):
    """A contiguous float32 CUDA tensor of shape (rows, N). numpy arrays and CPU tensors are
    copied to the current device; that copy is the caller's input transfer."""
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    if x.device.type != "cuda":
        x = x.to(device())
    if x.dtype != torch.float32:
        x = x.float()
    if not x.is_contiguous():
        x = x.contiguous()
    if x.dim() != 2 or (rows is not None and x.shape[0] != rows):
        raise ValueError(f"{name} must have shape ({rows if rows is not None else 'D'}, N); got {tuple(x.shape)}")
    return x


def as_actions(a, n, dev, name="action"):
    """An integer CUDA tensor of n elements (int32, int64 or uint8) and its ABI dtype code."""
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    if not isinstance(a, torch.Tensor):
        a = torch.as_tensor(a)
    if a.device != dev:
        a = a.to(dev)
    if a.dtype not in _DTYPES:
        if a.dtype.is_floating_point:
            raise ValueError(f"{name} must be an integer array, got {a.dtype}")
        a = a.to(torch.int64)
    if not a.is_contiguous():
        a = a.contiguous()
    if a.numel() != n:
        raise ValueError(f"{name} must have {n} elements; got {a.numel()}")
    return a, _DTYPES[a.dtype]


class PackedActions:
    """Actions packed along time for the CartPole and Acrobot step kernels (RLENV_U2): `bits` is a
    (ceil(steps / 4), N) uint8 tensor whose byte (r, i) holds environment i's actions of steps
    4r .. 4r + 3, step 4r + u in bits 2u; `steps` is T. Made by pack_actions; a quarter of the
    bytes of uint8 actions for a caller that streams them from host memory."""

    def __init__(self, bits, steps):
        self.bits = bits
        self.steps = int(steps)

    def checked(self, n, dev):
        """The bits as a contiguous uint8 tensor on dev, checked against T = steps and n."""
        b = torch.as_tensor(self.bits)
        rows = (self.steps + 3) // 4
        if b.dtype != torch.uint8 or self.steps < 0 or b.numel() != rows * n:
            raise ValueError(f"packed actions of {self.steps} steps and {n} environments must be uint8 "
                             f"({rows}, {n}); got {b.dtype} {tuple(b.shape)}")
        return b.to(dev).contiguous()


def pack_actions(a):
    """Actions (T, N) (or (N,) for one step) with values in 0..3, packed along time into
    PackedActions: byte (r, i) holds steps 4r .. 4r + 3 of environment i, two bits each, steps
    past T zero; on a's device."""
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    a = torch.as_tensor(a)
    if a.dtype.is_floating_point:
        raise ValueError(f"actions must be an integer array, got {a.dtype}")
    if a.dim() == 1:
        a = a[None]
    if a.dim() != 2:
        raise ValueError(f"actions must have shape (T, N) or (N,); got {tuple(a.shape)}")
    steps, n = a.shape
    b = a.to(torch.uint8) & 3
    pad = (-steps) % 4
    if pad:
        b = torch.cat([b, torch.zeros((pad, n), dtype=torch.uint8, device=b.device)])
    b = b.reshape(-1, 4, n)
    return PackedActions((b[:, 0] | (b[:, 1] << 2) | (b[:, 2] << 4) | (b[:, 3] << 6)).contiguous(), steps)


def step_outputs(rows, n, dev):
    """Fresh (next_state (rows, N) float32, reward (N,) float32, done (N,) bool), as MLX
    allocates a kernel's outputs per call."""
    return (torch.empty((rows, n), dtype=torch.float32, device=dev),
            torch.empty(n, dtype=torch.float32, device=dev),
            torch.empty(n, dtype=torch.bool, device=dev))


def ptr(t):
    return 0 if t is None else t.data_ptr()


def float_scalar(x):
    """A Python float from a float, a 0-d/1-element array or tensor."""
    if isinstance(x, torch.Tensor):
        return float(x.reshape(-1)[0].item())
    return float(np.asarray(x, dtype=np.float64).reshape(-1)[0])


class StepCounter:
    """The reference's per-call seed counter (`_calls`): incremented before every step, set
    by reseed (cartpole_metal.py:106-125)."""

    def __init__(self, start=0):
        self.calls = start

    def next(self, steps=1):
        first = self.calls + 1
        self.calls += steps
        return first & 0xFFFFFFFF


_reset_calls = 0


def next_reset_seed():
    """Seed for a `reset(n)` draw: a hash of a module-wide counter, kept apart from the small
    integers the step counters produce."""
    global _reset_calls
    _reset_calls += 1
    x = (_reset_calls * 0x9E3779B97F4A7C15 + 0x5EED) & 0xFFFFFFFFFFFFFFFF
    return ((x >> 32) ^ x) & 0xFFFFFFFF


def reset_uniform(rows, n, bound, center=None, seed=None, index_offset=0, dev=None):
    """(rows, n) float32 CUDA tensor: center + uniform in +-bound, drawn on the device."""
    dev = dev or device()
    out = torch.empty((rows, n), dtype=torch.float32, device=dev)
    c = None
    if center is not None:
        c = center if isinstance(center, torch.Tensor) else torch.as_tensor(np.asarray(center, dtype=np.float32))
        c = c.to(dev, torch.float32).contiguous()
    s = next_reset_seed() if seed is None else int(seed) & 0xFFFFFFFF
    check(lib().reset_uniform(out.data_ptr(), rows, n, ptr(c), bound, s, index_offset, stream_ptr(dev)))
    return out


def run_step_many(entry, rows, counter, state, actions, rewards=True, dones=True, sums=False, out=None):
    """Shared body of the `step_many` calls: T steps of one launch of `entry` (an ABI
    function with the rlenv_*_step_many signature) for actions (T, N), or PackedActions
    (CartPole and Acrobot only)."""
    state = as_state(state, rows)
    n, dev = state.shape[1], state.device
    if isinstance(actions, PackedActions):
        T = actions.steps
        actions, dt = actions.checked(n, dev), U2
    else:
        if not isinstance(actions, torch.Tensor):
            actions = torch.as_tensor(np.asarray(actions))
        if actions.dim() != 2 or actions.shape[1] != n:
            raise ValueError(f"actions must have shape (T, {n}); got {tuple(actions.shape)}")
        T = actions.shape[0]
        actions, dt = as_actions(actions, T * n, dev, "actions")
    final = torch.empty_like(state) if out is None else out
    rseq = torch.empty((T, n), dtype=torch.float32, device=dev) if rewards else None
    dseq = torch.empty((T, n), dtype=torch.bool, device=dev) if dones else None
    rsum = torch.empty(n, dtype=torch.float32, device=dev) if sums else None
    dcnt = torch.empty(n, dtype=torch.float32, device=dev) if sums else None
    check(entry(state.data_ptr(), actions.data_ptr(), dt, counter.next(T), T, n, 0, final.data_ptr(),
                ptr(rseq), ptr(dseq), ptr(rsum), ptr(dcnt), stream_ptr(dev)))
    return (final, rseq, dseq, rsum, dcnt) if sums else (final, rseq, dseq)


class StepBody:
    """Shared plumbing of the class-based drop-ins (Pendulum, Hopper, Legged): a per-instance
    call counter as the reference keeps (`self.calls`, pendulum_metal.py:118-123), fresh
    outputs per call, and the launch of one ABI step function."""

    rows = 0

    def __init__(self):
        self.calls = 0

    def reseed(self, seed=0):
        self.calls = seed

    def _next_seed(self):
        self.calls += 1
        return self.calls & 0xFFFFFFFF

    def _next_seeds(self, steps):
        """The first of `steps` consecutive per-call seeds, as `steps` single calls would draw them."""
        first = (self.calls + 1) & 0xFFFFFFFF
        self.calls += steps
        return first

    def _launch_many(self, entry, head, state, actions, tail=(), rewards=True, dones=True, extra=()):
        """entry(*head, state, actions, dtype, seed0, *tail, steps, n, index_offset, state_out,
        reward_seq, done_seq, *extra, stream) for actions (T, N): T steps in one launch, equal to T
        `step` calls. `extra` are further output tensors passed after done_seq. Returns
        (final_state, rewards (T, N) or None, dones (T, N) or None, *extra)."""
        state = as_state(state, self.rows)
        n, dev = state.shape[1], state.device
        if not isinstance(actions, torch.Tensor):
            actions = torch.as_tensor(np.asarray(actions))
        if actions.dim() != 2 or actions.shape[1] != n:
            raise ValueError(f"actions must have shape (T, {n}); got {tuple(actions.shape)}")
        steps = actions.shape[0]
        actions, dt = as_actions(actions, steps * n, dev, "actions")
        final = torch.empty_like(state)
        rseq = torch.empty((steps, n), dtype=torch.float32, device=dev) if rewards else None
        dseq = torch.empty((steps, n), dtype=torch.bool, device=dev) if dones else None
        check(entry(*head, state.data_ptr(), actions.data_ptr(), dt, self._next_seeds(steps), *tail, steps, n, 0,
                    final.data_ptr(), ptr(rseq), ptr(dseq), *(ptr(x) for x in extra), stream_ptr(dev)))
        return (final, rseq, dseq, *extra)

    def _launch(self, entry, head, state, action, tail=(), outs=()):
        """entry(*head, state, action, dtype, seed, *tail, n, index_offset, next, reward, done,
        *outs, stream); outs are raw device pointers (or None) of further outputs."""
        state = as_state(state, self.rows)
        n = state.shape[1]
        action, dt = as_actions(action, n, state.device)
        nxt, reward, done = step_outputs(self.rows, n, state.device)
        check(entry(*head, state.data_ptr(), action.data_ptr(), dt, self._next_seed(), *tail, n, 0,
                    nxt.data_ptr(), reward.data_ptr(), done.data_ptr(), *outs, stream_ptr(state.device)))
        return nxt, reward, done


def as_theta(theta, p, d, dev):
    """theta_pop (P, D) float32 contiguous on dev and its row stride; a single row (D,) or
    (1, D) is shared by every member (stride 0)."""
    if isinstance(theta, np.ndarray):
        theta = torch.from_numpy(np.ascontiguousarray(theta))
    if not isinstance(theta, torch.Tensor):
        theta = torch.as_tensor(theta)
    theta = theta.to(dev, torch.float32)
    if theta.dim() == 1 or (theta.dim() == 2 and theta.shape[0] == 1 and p != 1):
        theta = theta.reshape(1, -1).contiguous()
        stride = 0
    else:
        theta = theta.contiguous()
        stride = theta.shape[1] if theta.dim() == 2 else -1
        if theta.dim() != 2 or theta.shape[0] != p:
            raise ValueError(f"theta_pop must have shape ({p}, {d}) or ({d},); got {tuple(theta.shape)}")
    if theta.shape[-1] != d:
        raise ValueError(f"theta_pop rows must have {d} parameters for this hidden width; got {theta.shape[-1]}")
    return theta, stride
