"""Trusted evaluation: ``evaluate_bpb`` and ``causality_check`` with the reference's
signatures and return contracts (``prepare.py:591-684``).

bpb = total nats over tokens with a positive byte length / (ln 2 * total bytes of
valid tokens); the CE is computed here, in fp32, from the model's logits
(``model(x)`` must return softcapped logits), never by calling ``model(x, y)``.
Per-rank token cap ``ceil(max_tokens / world)``; three SUM all-reduces of the
scalars across ranks.
"""
from __future__ import annotations

import math
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .config import EVAL_TIMEOUT_SECONDS, TOKENIZER_VOCAB_SIZE
from .data import synthetic as syn
from .data.loader import make_eval_dataloader


class EvalTimeoutError(TimeoutError):
    pass


@torch.no_grad()
def evaluate_bpb(model: torch.nn.Module, tokenizer, batch_size: int, seq_len: int, device,
                 split: str = "public_val", max_tokens: int | None = None,
                 timeout_seconds: int = EVAL_TIMEOUT_SECONDS, shard_ids=None,
                 stream_tokens: int | None = None) -> dict:
    started = time.monotonic()
    dev = torch.device(device)
    vocab = tokenizer.get_vocab_size() if tokenizer is not None else TOKENIZER_VOCAB_SIZE
    # a text tokenizer's UTF-8 byte table, else the synthetic corpus's
    token_bytes = (tokenizer.token_bytes().to(dev) if hasattr(tokenizer, "token_bytes")
                   else syn.get_token_bytes(dev, vocab))
    world_size = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    limit = None if max_tokens is None else max(1, math.ceil(max_tokens / max(world_size, 1)))
    n_stream = stream_tokens or (max_tokens + world_size * (seq_len + 1) if max_tokens else 1 << 21)
    loader = make_eval_dataloader(tokenizer, batch_size, seq_len, split, dev, max_stream_tokens=n_stream)
    model.eval()
    total_nats = torch.tensor(0.0, dtype=torch.float32, device=dev)
    total_bytes = torch.tensor(0, dtype=torch.int64, device=dev)
    total_tokens = torch.tensor(0, dtype=torch.int64, device=dev)
    local_tokens = 0
    for x, y, _ in loader:
        if time.monotonic() - started > timeout_seconds:
            raise EvalTimeoutError(f"evaluation exceeded {timeout_seconds}s")
        logits = model(x)
        if logits.size(-1) < vocab:
            raise RuntimeError(f"model vocab too small: {logits.size(-1)} < {vocab}")
        logits = logits[..., :vocab].float()
        loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), y.reshape(-1), ignore_index=-1, reduction="none")
        y_flat = y.reshape(-1)
        valid = y_flat >= 0
        nbytes = token_bytes[y_flat.clamp_min(0)]
        mask = valid & (nbytes > 0)
        total_nats += (loss * mask).sum()
        total_bytes += (nbytes * valid).sum()
        bt = valid.sum()
        total_tokens += bt
        local_tokens += int(bt.item())
        if limit is not None and local_tokens >= limit:
            break
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(total_nats, op=dist.ReduceOp.SUM)
        dist.all_reduce(total_bytes, op=dist.ReduceOp.SUM)
        dist.all_reduce(total_tokens, op=dist.ReduceOp.SUM)
    elapsed = time.monotonic() - started
    nats = total_nats.item()
    nb = int(total_bytes.item())
    bpb = nats / (math.log(2) * nb) if nb > 0 else float("inf")
    return {"val_bpb": float(bpb), "eval_seconds": float(elapsed), "eval_timeout": int(timeout_seconds),
            "eval_over_timeout": bool(elapsed > timeout_seconds), "num_tokens": int(total_tokens.item()),
            "num_bytes": nb, "total_nats": float(nats)}


@torch.no_grad()
def causality_check(model: torch.nn.Module, tokenizer, batch_size: int, seq_len: int, device,
                    tolerance: float = 1e-2, split: str = "public_val", shard_ids=None) -> dict:
    """Future tokens must not change earlier logits: reverse the second half of a batch
    and require logits before ``cut - 1`` to move by at most ``tolerance``."""
    dev = torch.device(device)
    loader = make_eval_dataloader(tokenizer, batch_size, seq_len, split, dev,
                                  max_stream_tokens=batch_size * (seq_len + 1) * 2)
    x, _y, _ = next(loader)
    cut = max(2, seq_len // 2)
    x2 = x.clone()
    x2[:, cut:] = torch.flip(x2[:, cut:], dims=[1])
    model.eval()
    a = model(x)[:, :cut - 1].float()
    b = model(x2)[:, :cut - 1].float()
    max_abs = (a - b).abs().max().item()
    return {"passed": bool(max_abs <= tolerance), "max_abs_diff": float(max_abs), "tolerance": tolerance}
