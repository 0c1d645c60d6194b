"""Data-parallel gradient plumbing with the reference's helper API
(``train.py:4383-4528``): per-parameter ``sync_gradients`` (the NCCL baseline),
flat-buffer ``build_flat_grad_buffer`` / ``sync_gradients_flat`` /
``clip_grad_norm_flat_``, dynamic loss scaling helpers and the clip split.

The engine's own paths (bucketed all-reduce overlapped with backward, distributed
Muon, fused NVLink kernels) live in ``parallel.buckets`` / ``parallel.dist_muon`` and
reuse the flat-buffer layout built here.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..runtime import is_dist


def split_clip_params(model, exclude_ngram: bool = True):
    """(main, ngram) parameter lists for clipping: hashed n-gram / output-bigram tables
    get their own norm so they do not rescale every other tensor's update."""
    ids = set()
    if exclude_ngram:
        ids = {id(p) for p in model.ngram_embeds.parameters()}
        if getattr(model, "out_bigram", None) is not None:
            ids.add(id(model.out_bigram.weight))
        if getattr(model, "engram", None) is not None:
            ids |= {id(p) for p in model.engram.tables.parameters()}
    if not ids:
        return list(model.parameters()), []
    main, ng = [], []
    for p in model.parameters():
        (ng if id(p) in ids else main).append(p)
    return main, ng


def sync_gradients(model, skip_param_ids: frozenset[int] | None = None) -> None:
    """Per-parameter all_reduce(AVG): the reference's synchronous NCCL path."""
    if not is_dist():
        return
    for p in model.parameters():
        if p.grad is not None and not (skip_param_ids and id(p) in skip_param_ids):
            dist.all_reduce(p.grad, op=dist.ReduceOp.AVG)


def build_flat_grad_buffer(model) -> tuple[torch.Tensor, list[torch.Tensor]]:
    params = [p for p in model.parameters() if p.requires_grad]
    device = params[0].device if params else torch.device("cpu")
    total = sum(p.numel() for p in params)
    flat = torch.zeros(total, dtype=torch.float32, device=device)
    off = 0
    for p in params:
        n = p.numel()
        p.grad = flat[off:off + n].view_as(p)
        off += n
    return flat, params


def sync_gradients_flat(flat: torch.Tensor) -> None:
    if is_dist():
        dist.all_reduce(flat, op=dist.ReduceOp.AVG)


def clip_grad_norm_flat_(flat: torch.Tensor, max_norm: float) -> torch.Tensor:
    total = flat.norm(2)
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    flat.mul_(coef)
    return total


def loss_scale_transition(scale: float, clean: int, finite: bool, growth_interval: int, max_scale: float):
    """One dynamic-loss-scaling step: halve + skip on overflow, double every
    ``growth_interval`` clean steps (capped).  Returns (scale, clean, skip)."""
    if not finite:
        return (max(1.0, scale / 2.0), 0, True)
    clean += 1
    if clean >= growth_interval and scale < max_scale:
        return (min(max_scale, scale * 2.0), 0, False)
    return (scale, clean, False)


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
