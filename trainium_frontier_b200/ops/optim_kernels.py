"""Python front-end of the optimizer kernels (``csrc/kernels/optim_kernels.cu``).

Reference counterpart: the foreach AdamW / RMSProp of ``MuonAdamW`` (``train.py:3961-4127``).
"""
from __future__ import annotations

import torch

from ._ext import C


def adamw_multi(params, grads, exp_avgs, exp_avg_sqs, lr: torch.Tensor, beta1: float, beta2: float,
                eps: float, wd: float, bias1, bias2, cautious: bool = False) -> None:
    """One multi-tensor launch for a whole AdamW group (fp32 params / grads / moments)."""
    grads = [g if g.dtype == torch.float32 and g.is_contiguous() else g.float().contiguous() for g in grads]
    C().adamw_multi([p.data for p in params], grads, exp_avgs, exp_avg_sqs, lr, float(beta1), float(beta2),
                    float(eps), float(wd), [float(b) for b in bias1], [float(b) for b in bias2], bool(cautious))


def muon_apply(w: torch.Tensor, g: torch.Tensor, lr: torch.Tensor, lrwd: torch.Tensor, params=None) -> None:
    """w -= bf16(lr) * g + lrwd * w * [g * w >= 0] in place (fp32 w, bf16 g)."""
    C().muon_apply(w, g.contiguous(), lr.reshape(1).contiguous(), lrwd.reshape(1).contiguous())
