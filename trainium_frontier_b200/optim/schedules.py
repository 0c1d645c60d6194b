"""Learning-rate / momentum / weight-decay / beta schedules (reference
``train.py:4749-4928`` and the per-step group rewrite at ``train.py:6089-6119``).

Progress is the fraction of the run elapsed.  The reference keys it on wall clock
(elapsed / max_train_seconds); ``progress_mode="steps"`` keys it on step / num_steps
instead, which makes two runs comparable step for step (used by parity tests and the
benchmark, where wall-clock noise would otherwise change the schedule).
"""
from __future__ import annotations

from ..config import RunConfig, parse_float_tuple, parse_int_tuple


def lr_multiplier(cfg: RunConfig, step: int, progress: float) -> float:
    if step < cfg.warmup_steps:
        return (step + 1) / max(1, cfg.warmup_steps)
    if cfg.warmdown_ratio <= 0.0:
        return 1.0
    progress = min(1.0, max(0.0, progress))
    if progress < 1.0 - cfg.warmdown_ratio:
        return 1.0
    cooldown = (1.0 - progress) / cfg.warmdown_ratio
    lrm = cooldown * 1.0 + (1 - cooldown) * cfg.final_lr_frac
    if cfg.lrm_quantum > 0:
        lrm = round(lrm * cfg.lrm_quantum) / cfg.lrm_quantum
    return lrm


def lr_flat_multiplier(cfg: RunConfig, step: int) -> float:
    """Warmup-only multiplier for groups with ``no_lr_decay`` (hashed n-gram tables)."""
    return min(1.0, (step + 1) / max(1, cfg.warmup_steps))


def muon_momentum(cfg: RunConfig, step: int, progress: float = 0.0) -> float:
    """0.85 -> 0.95 over ``muon_momentum_warmup_steps``, then an optional cooldown back
    down over the last ``muon_momentum_cooldown_frac`` of the run."""
    frac = min(step / max(1, cfg.muon_momentum_warmup_steps), 1.0)
    m = (1 - frac) * 0.85 + frac * 0.95
    if cfg.muon_momentum_cooldown_frac > 0.0:
        cd = min(1.0, max(0.0, (progress - (1.0 - cfg.muon_momentum_cooldown_frac))
                          / cfg.muon_momentum_cooldown_frac))
        m = (1 - cd) * m + cd * cfg.muon_momentum_final
    return m


def muon_weight_decay(cfg: RunConfig, progress: float) -> float:
    return cfg.weight_decay * (1.0 - min(1.0, progress)) if cfg.wd_decay_to_zero else cfg.weight_decay


def demon_beta1_scale(cfg: RunConfig, progress: float) -> float:
    if not cfg.demon_beta1:
        return 1.0
    start = cfg.demon_beta1_start_frac if cfg.demon_beta1_start_frac >= 0.0 else (1.0 - cfg.warmdown_ratio)
    start = min(max(start, 0.0), 0.999)
    frac = min(1.0, max(0.0, (progress - start) / max(1e-6, 1.0 - start)))
    return 1.0 + frac * (cfg.demon_beta1_final / cfg.demon_beta1_ref - 1.0)


def muon_beta2(cfg: RunConfig, progress: float) -> float:
    if cfg.muon_beta2_final <= 0.0:
        return cfg.muon_beta2
    p = min(1.0, max(0.0, progress))
    return cfg.muon_beta2 + p * (cfg.muon_beta2_final - cfg.muon_beta2)


def muon_depth_mults(cfg: RunConfig, depths: list[int | None], n_layer: int) -> tuple[list[float], list[float]]:
    """Per-parameter (lr multiplier, (1 - momentum) multiplier), linear in depth."""
    lr_on = not (cfg.muon_depth_lr_bottom == 1.0 and cfg.muon_depth_lr_top == 1.0)
    mom_on = cfg.muon_depth_mom_bottom > 0.0 and cfg.muon_depth_mom_top > 0.0
    span = max(1, n_layer - 1)
    lr_mult, mom_mult = [], []
    for d in depths:
        if d is None or not lr_on:
            lr_mult.append(1.0)
        else:
            f = d / span
            lr_mult.append(cfg.muon_depth_lr_bottom + f * (cfg.muon_depth_lr_top - cfg.muon_depth_lr_bottom))
        if d is None or not mom_on:
            mom_mult.append(1.0)
        else:
            f = d / span
            target = cfg.muon_depth_mom_bottom + f * (cfg.muon_depth_mom_top - cfg.muon_depth_mom_bottom)
            mom_mult.append((1.0 - target) / max(1e-6, 1.0 - cfg.muon_depth_mom_ref))
    return lr_mult, mom_mult


def batch_ramp_stage(cfg: RunConfig, progress: float) -> int:
    lo, hi = parse_float_tuple(cfg.batch_ramp_bounds)
    if progress < lo:
        return 0
    if progress < hi:
        return 1
    return 2


def batch_ramp_grad_accum(cfg: RunConfig, progress: float, grad_accum_ref: int) -> tuple[int, float]:
    if not cfg.batch_ramp:
        return grad_accum_ref, 1.0
    gas = parse_int_tuple(cfg.batch_ramp_grad_accum)[batch_ramp_stage(cfg, progress)]
    return gas, (gas / grad_accum_ref) ** cfg.batch_ramp_lr_exp


def apply_schedules(cfg: RunConfig, optimizer, step: int, progress: float, batch_lr_scale: float = 1.0) -> float:
    """Rewrite every param group's lr / momentum / weight decay / betas for this step."""
    lrm = lr_multiplier(cfg, step, progress)
    lrm_flat = lr_flat_multiplier(cfg, step)
    db1 = demon_beta1_scale(cfg, progress)
    mb2 = muon_beta2(cfg, progress)
    for group in optimizer.param_groups:
        group["lr"] = group["initial_lr"] * batch_lr_scale * (lrm_flat if group.get("no_lr_decay") else lrm)
        if group["kind"] == "muon":
            group["momentum"] = muon_momentum(cfg, step, progress)
            group["weight_decay"] = muon_weight_decay(cfg, progress)
            group["beta2"] = mb2
        elif group["kind"] == "adamw" and cfg.demon_beta1:
            b1, b2 = group["initial_betas"]
            group["betas"] = (b1 * db1, b2)
    return lrm
