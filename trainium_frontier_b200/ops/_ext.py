"""Loader of the compiled sm_100a kernel module ``trainium_frontier_b200._C``.

CUDA tensors always run through these kernels: if the in-tree extension is missing
on a machine with a GPU, ``C()`` raises instead of falling back to a library path.
CPU tensors never reach this module (the ops' CPU branch is the fp32 oracle).
"""
from __future__ import annotations

import importlib

import torch

_C = None
_ERR: dict[int, torch.Tensor] = {}
_LAUNCHES = [0]
_BY_NAME: dict[str, int] = {}


class _Counted:
    """Proxy over the extension module that counts kernel-launching calls."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*a, **k):
            _LAUNCHES[0] += 1
            _BY_NAME[name] = _BY_NAME.get(name, 0) + 1
            return fn(*a, **k)
        return wrapped


def C():
    global _C
    if _C is None:
        try:
            _C = _Counted(importlib.import_module("trainium_frontier_b200._C"))
        except ImportError as e:
            raise ImportError(
                "trainium_frontier_b200._C (sm_100a kernels) is not built. Run "
                "`python setup.py build_ext --inplace` at the repository root.") from e
    return _C


def launch_count() -> int:
    """Number of sm_100a kernel launches issued through ``C()`` so far."""
    return _LAUNCHES[0]


def launch_counts_by_name() -> dict[str, int]:
    """Kernel-launching calls through ``C()`` so far, per entry point name (a copy)."""
    return dict(_BY_NAME)


def available() -> bool:
    try:
        C()
        return True
    except ImportError:
        return False


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word that every bounded wait in the kernels reports into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = t
    return t


class KernelTimeout(RuntimeError):
    pass


def check_errors(device: torch.device | None = None, reset: bool = True) -> int:
    """Read the device error word (synchronizes); raise if a kernel gave up waiting."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    t = err_word(dev)
    v = int(t.item())
    if v and reset:
        t.zero_()
    if v:
        raise KernelTimeout(f"a kernel reported error code {v:#x} (bounded wait ran out)")
    return v
