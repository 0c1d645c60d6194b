"""Flash attention front-end (``csrc/kernels/attention_sm100.cu``).

``flash_fwd`` / ``flash_bwd`` take row views ``[B*T, >= H*D]`` whose head ``h`` lives in
columns ``[h*D, h*D + D)`` -- exactly the fused projection buffers -- so no
transposes or copies are made on the way in or out.  Requirements: T % 128 == 0,
head_dim in {64, 128}.

Reference counterparts: the SDPA call of ``CausalSelfAttention`` (``train.py:2564-2567``)
and the research NKI kernels it never shipped (``research/scratch/nki_attn_fwd.py:41-132``,
``research/scratch/nki_attn_bwd.py:1-367``).
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from ._ext import C, err_word


def supported(T: int, D: int) -> bool:
    return T % 128 == 0 and D in (64, 128)


def flash_fwd(q, k, v, B, T, H, D, scale, causal=True, out=None):
    M = B * T
    if out is None:
        out = torch.empty((M, H * D), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B * H * T, dtype=torch.float32, device=q.device)
    C().fa_fwd(q, k, v, B, T, H, D, float(scale), bool(causal), out, lse, err_word(q.device))
    return out, lse


def flash_bwd(q, k, v, o, dout, lse, B, T, H, D, scale, causal=True, dq=None, dk=None, dv=None):
    M = B * T
    dev = q.device
    if dq is None:
        dq = torch.empty((M, H * D), dtype=torch.bfloat16, device=dev)
    if dk is None:
        dk = torch.empty((M, H * D), dtype=torch.bfloat16, device=dev)
    if dv is None:
        dv = torch.empty((M, H * D), dtype=torch.bfloat16, device=dev)
    dq_acc = torch.empty((M, H * D), dtype=torch.float32, device=dev)
    dvec = torch.empty(B * H * T, dtype=torch.float32, device=dev)
    C().fa_bwd(q, k, v, o, dout, lse, B, T, H, D, float(scale), bool(causal), dq_acc, dq, dk, dv, dvec,
               err_word(dev))
    return dq, dk, dv


class FlashAttnFn(Function):
    """Attention over q, k, v [B, T, H, D] (any strides with a unit inner one)."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        B, T, H, D = q.shape
        q2, k2, v2 = (t.contiguous().view(B * T, H * D) for t in (q, k, v))
        o, lse = flash_fwd(q2, k2, v2, B, T, H, D, scale, causal)
        ctx.save_for_backward(q2, k2, v2, o, lse)
        ctx.meta = (B, T, H, D, scale, causal)
        return o.view(B, T, H, D)

    @staticmethod
    def backward(ctx, do):
        q2, k2, v2, o, lse = ctx.saved_tensors
        B, T, H, D, scale, causal = ctx.meta
        dq, dk, dv = flash_bwd(q2, k2, v2, o, do.contiguous().view(B * T, H * D), lse, B, T, H, D, scale, causal)
        return dq.view(B, T, H, D), dk.view(B, T, H, D), dv.view(B, T, H, D), None, None
