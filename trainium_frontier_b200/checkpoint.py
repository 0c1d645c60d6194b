"""``out/final.pt`` writer / reader with the reference payload layout
(``train.py:4660-4743``): ``{"model_state", "model_config", "toggles", "meta"
[, "ema_state"]}``, tensors on CPU, loadable with ``torch.load(weights_only=True)``.

``load_for_eval(path, device)`` keeps the two-argument scoring contract: it rebuilds
``GPT(GPTConfig(**model_config))`` with ``sequence_len >= 8192`` (rotary tables are
not parameters), strict-loads (preferring EMA weights when present) and returns the
model in eval mode.  Unlike the reference, the architecture toggles are read back from
the checkpoint's own ``toggles`` entry, so a checkpoint is self-describing.

Full resume (an extension; the reference only warm-starts) stores optimizer state,
step counters, RNG states and the loader position next to the final checkpoint.
"""
from __future__ import annotations

import dataclasses
import os
from pathlib import Path

import torch

from .config import EVAL_MIN_SEQ_LEN, GPTConfig, RunConfig, SHAPE_CRITICAL_TOGGLES
from .runtime import compute_dtype_for, print0


def torch_load_weights(path, map_location):
    return torch.load(path, map_location=map_location, weights_only=True)


def save_checkpoint(path, model, meta: dict, ema_state: dict | None = None, toggles: dict | None = None) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    rc = getattr(model, "rc", None)
    payload = {
        "model_state": {k: v.detach().to("cpu", copy=True).contiguous() for k, v in model.state_dict().items()},
        "model_config": dataclasses.asdict(model.config),
        "toggles": toggles if toggles is not None else (rc.toggles() if rc is not None else {}),
        "meta": meta,
    }
    if ema_state is not None:
        payload["ema_state"] = {k: v.detach().to("cpu", copy=True) for k, v in ema_state.items()}
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(payload, tmp)
    os.replace(tmp, path)


def _rc_from_toggles(toggles: dict, base: RunConfig | None = None) -> RunConfig:
    base = base or RunConfig()
    names = {f.name for f in dataclasses.fields(RunConfig)}
    kw = {k: v for k, v in (toggles or {}).items() if k in names}
    return dataclasses.replace(base, **kw)


def warm_start_from(path, model) -> dict:
    """Load weights into a freshly built model (fresh optimizer, step 0)."""
    payload = torch_load_weights(path, map_location="cpu")
    saved = payload.get("toggles", {})
    rc = getattr(model, "rc", None)
    live = rc.toggles() if rc is not None else {}
    for k in saved:
        if k in live and saved[k] != live[k]:
            tag = "SHAPE-CRITICAL" if k in SHAPE_CRITICAL_TOGGLES else "silent-behavior"
            print0(f"WARNING [{tag}]: toggle {k} mismatch -- checkpoint={saved[k]!r} current={live[k]!r}")
    with torch.no_grad():
        model.load_state_dict(payload["model_state"], strict=True)
    meta = payload.get("meta", {})
    print0(f"warm-started from {path}: step={meta.get('step')} tokens={meta.get('total_train_tokens')}")
    return meta


def load_for_eval(checkpoint_path, device, prefer_ema: bool = True):
    from .models.gpt import GPT
    device = torch.device(device)
    payload = torch_load_weights(checkpoint_path, map_location="cpu")
    config = GPTConfig(**payload["model_config"])
    if config.sequence_len < EVAL_MIN_SEQ_LEN:
        config.sequence_len = EVAL_MIN_SEQ_LEN
    rc = _rc_from_toggles(payload.get("toggles", {}))
    model = GPT(config, rc)
    model.set_compute_dtype(compute_dtype_for(device))
    model.init_weights()
    state = payload["model_state"]
    if prefer_ema and "ema_state" in payload and os.environ.get("NEURON_COMPETITION_R1_EVAL_PREFER_EMA", "1") != "0":
        state = payload["ema_state"]
    model.load_state_dict(state, strict=True)
    model.to(device)
    model.eval()
    return model


def save_resume(path, optimizer, step: int, extra: dict) -> None:
    """Optimizer state + counters + RNG for an exact continuation."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    payload = {
        "optimizer": optimizer.state_dict(),
        "step": step,
        "rng_cpu": torch.get_rng_state(),
        "rng_cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else [],
        "extra": extra,
    }
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(payload, tmp)
    os.replace(tmp, path)


def load_resume(path, optimizer) -> dict:
    payload = torch.load(path, map_location="cpu", weights_only=False)
    optimizer.load_state_dict(payload["optimizer"])
    torch.set_rng_state(payload["rng_cpu"])
    if torch.cuda.is_available() and payload.get("rng_cuda"):
        try:
            torch.cuda.set_rng_state_all(payload["rng_cuda"])
        except Exception:
            pass
    return payload
