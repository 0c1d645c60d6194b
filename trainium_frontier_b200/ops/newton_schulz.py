"""Batched Polar-Express Newton-Schulz orthogonalisation of stacked matrices.

For X [K, r, c] (already Frobenius-normalised), five iterations of
    wide (r <= c):  S = X X^T ;  M = b S + c S^2 ;  X <- a X + M X
    tall (r >  c):  S = X^T X ;  M = b S + c S^2 ;  X <- a X + X M
(reference ``train.py:3629-3636``).  On the GPU each iteration is three batched
tcgen05 GEMMs with the polynomial folded into the epilogues: the second GEMM writes
``c * (S @ S) + b * S`` and the third ``a * X + (M @ X)`` directly, so no elementwise
pass touches HBM between them.  On the CPU it is the reference's own matmul chain.
"""
from __future__ import annotations

import torch

from ..config import POLAR_EXPRESS_COEFFS


def newton_schulz_reference(x: torch.Tensor, steps: int) -> torch.Tensor:
    if x.shape[-2] > x.shape[-1]:
        for a, b, c in POLAR_EXPRESS_COEFFS[:steps]:
            xtx = x.mT @ x
            x = a * x + x @ (b * xtx + c * (xtx @ xtx))
    else:
        for a, b, c in POLAR_EXPRESS_COEFFS[:steps]:
            xxt = x @ x.mT
            x = a * x + (b * xxt + c * (xxt @ xxt)) @ x
    return x


def newton_schulz_gpu(x: torch.Tensor, steps: int) -> torch.Tensor:
    from . import gemm
    squeeze = x.dim() == 2
    if squeeze:
        x = x.unsqueeze(0)
    x = x.contiguous()
    K, r, c = x.shape
    tall = r > c
    n = c if tall else r
    S = torch.empty((K, n, n), dtype=torch.bfloat16, device=x.device)
    Mt = torch.empty_like(S)
    y = torch.empty_like(x)
    for a, b, cc in POLAR_EXPRESS_COEFFS[:steps]:
        if tall:
            gemm.bmm_tn(x, x, S)                                   # S = X^T X
        else:
            gemm.bmm_nt(x, x, S)                                   # S = X X^T
        gemm.bmm_nt(S, S, Mt, residual=S, alpha=cc, rcoef=b)       # M = c S S^T + b S  (S symmetric)
        if tall:
            gemm.bmm_nt(x, Mt, y, residual=x, alpha=1.0, rcoef=a)  # X M  (M symmetric)
        else:
            gemm.bmm_nn(Mt, x, y, residual=x, alpha=1.0, rcoef=a)  # M X
        x, y = y, x
    return x.squeeze(0) if squeeze else x


def newton_schulz(x: torch.Tensor, steps: int) -> torch.Tensor:
    from . import oracle_active
    if x.is_cuda and x.dtype == torch.bfloat16 and not oracle_active():
        return newton_schulz_gpu(x, steps)
    return newton_schulz_reference(x, steps)
