"""Python front-end of the optimizer kernels (``csrc/kernels/optim_kernels.cu``).

Reference counterparts: the foreach AdamW / RMSProp of ``MuonAdamW`` (``train.py:3961-4127``)
and the Muon math of one stack (``train.py:3574-3647``).
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


def muon_stack_fusable(g, mb, mom, lr) -> bool:
    """The fused owner path takes fp32 contiguous [K, r, c] gradient / momentum stacks and
    0-dim (per-group) momentum and learning-rate scalars."""
    return (g.is_cuda and g.dim() == 3 and g.dtype == torch.float32 and g.is_contiguous()
            and mb.dtype == torch.float32 and mb.is_contiguous() and mom.dim() == 0 and lr.dim() == 0
            and (g.shape[-1] * g.shape[-2]) % 8 == 0 and g.shape[-1] % 8 == 0)


def muon_owner_update(g: torch.Tensor, mb: torch.Tensor, second: torch.Tensor, mom: torch.Tensor,
                      one_mom: torch.Tensor, one_b2: torch.Tensor, ns_steps: int, coef: torch.Tensor | None = None,
                      out: torch.Tensor | None = None, w: torch.Tensor | None = None,
                      lr: torch.Tensor | None = None, lrwd: torch.Tensor | None = None) -> None:
    """Muon on one stack [K, r, c] in six launches plus the Newton-Schulz GEMMs: momentum /
    Nesterov / bf16 / sum of squares (``muon_pre``), Frobenius normalisation, Newton-Schulz,
    NorMuon second moment and scale; the scaled bf16 update goes to ``out``, or is applied
    to the fp32 masters ``w`` with ``lr`` / ``lrwd`` (device scalars)."""
    from . import newton_schulz as ns
    K = g.shape[0]
    x = torch.empty(g.shape, dtype=torch.bfloat16, device=g.device)
    fro = torch.empty(K, 64, dtype=torch.float32, device=g.device)  # per-block partial sums (fixed order)
    C().muon_pre(g, mb, x, None if coef is None else coef.reshape(1), mom.reshape(1), one_mom.reshape(1), fro)
    C().muon_fro_scale(x, fro)
    gq = ns.newton_schulz(x, ns_steps)
    C().normuon_tail(gq, second, one_b2.reshape(1), out, w, None if lr is None else lr.reshape(1),
                     None if lrwd is None else lrwd.reshape(1))
