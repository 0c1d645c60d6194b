"""trainium_frontier_b200: a B200-native (sm_100a) small-GPT pretraining framework.

Layers (bottom-up): ``runtime`` (process/device), ``data`` (synthetic corpus, packing
loaders), ``ops`` (tcgen05/TMA/TMEM kernels + their autograd wrappers), ``models``
(the GPT family), ``optim`` (MuonAdamW + schedules), ``parallel`` (DP gradient sync,
distributed Muon, fused NVLink kernels, tensor parallelism), ``eval`` / ``checkpoint``
(scoring contract and ``out/final.pt``), ``inference`` (KV-cache decode) and
``train`` (the CLI entry point).
"""
from __future__ import annotations

import importlib

__version__ = "0.1.0"

_NATIVE = None


def _native_ext():
    """The host C++ runtime extension (data loader).  Raises a clear error when the
    in-tree build is missing instead of silently using a slow path."""
    global _NATIVE
    if _NATIVE is None:
        try:
            _NATIVE = importlib.import_module("trainium_frontier_b200._native")
        except ImportError as e:  # pragma: no cover - exercised only on a broken build
            raise ImportError(
                "trainium_frontier_b200._native is not built; run "
                "`python setup.py build_ext --inplace` at the repository root") from e
    return _NATIVE
