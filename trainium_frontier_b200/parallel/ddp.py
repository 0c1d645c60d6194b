"""Data-parallel gradient helpers used around the engine's own sync paths.

* ``sync_gradients`` is the per-parameter ``all_reduce(AVG)`` baseline the reference
  uses on CUDA (``train.py:4412-4420``); the engine keeps it as its ``per_param`` mode.
* Dynamic loss scaling (``train.py:4493-4528``): ``next_loss_scale`` decides the next
  scale from whether this step's gradients were finite; ``grads_finite_`` and
  ``unscale_grads_`` work on the engine's flat fp32 gradient buffer.

The engine's other modes (bucketed all-reduce overlapped with backward, distributed
Muon over NCCL, the fused NVLink kernels) live in ``engine`` and ``parallel.dist_muon``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..runtime import is_dist


def sync_gradients(model, skip_param_ids: frozenset[int] | None = None) -> None:
    """Per-parameter all_reduce(AVG): the reference's synchronous NCCL path."""
    if not is_dist():
        return
    for p in model.parameters():
        if p.grad is not None and not (skip_param_ids and id(p) in skip_param_ids):
            dist.all_reduce(p.grad, op=dist.ReduceOp.AVG)


def next_loss_scale(scale: float, clean_steps: int, finite: bool, growth_interval: int,
                    max_scale: float) -> tuple[float, int, bool]:
    """Dynamic loss scale after one step.  Returns ``(scale, clean_steps, skip_step)``.

    A step whose gradients overflowed is skipped and the scale halves (never below 1);
    otherwise the run of clean steps grows, and once it reaches ``growth_interval`` the
    scale doubles (capped at ``max_scale``) and the run restarts."""
    if not finite:
        return max(scale * 0.5, 1.0), 0, True
    run = clean_steps + 1
    grow = run >= growth_interval and scale < max_scale
    return (min(scale * 2.0, max_scale) if grow else scale), (0 if grow else run), False


def grads_finite_(model, flat: torch.Tensor | None) -> bool:
    if flat is not None:
        return bool(torch.isfinite(flat).all().item())
    for p in model.parameters():
        if p.grad is not None and not bool(torch.isfinite(p.grad).all().item()):
            return False
    return True


def unscale_grads_(model, flat: torch.Tensor | None, scale: float) -> None:
    if scale == 1.0:
        return
    if flat is not None:
        flat.div_(scale)
        return
    for p in model.parameters():
        if p.grad is not None:
            p.grad.div_(scale)
