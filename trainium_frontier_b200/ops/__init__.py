"""Public op surface of the framework.

Every op has two implementations selected by the device of its inputs:
* CUDA tensors -> the hand-written sm_100a kernels (``ops.fused`` over ``_C``); the
  extension is required there and its absence raises.
* CPU tensors  -> the fp32 PyTorch oracle in ``ops.reference`` (reference op order),
  which is also what the GPU numerics tests compare against.

``oracle_mode()`` routes CUDA tensors through the oracle as well (library GEMMs, SDPA,
eager elementwise ops in the compute dtype): the bf16 library comparator of the
benchmark runs the same model and engine that way.  It is a measurement switch, never
the training path.
"""
from __future__ import annotations

import contextlib
import os

import torch

from . import reference as ref

_ORACLE = [False]


@contextlib.contextmanager
def oracle_mode(on: bool = True):
    """Within the block, every op (and the optimizer's kernel paths) uses the PyTorch
    oracle on any device."""
    prev = _ORACLE[0]
    _ORACLE[0] = bool(on)
    try:
        yield
    finally:
        _ORACLE[0] = prev


def oracle_active() -> bool:
    return _ORACLE[0]


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda and not _ORACLE[0]


def norm(x: torch.Tensor) -> torch.Tensor:
    if _cuda(x):
        from .fused import RMSNormFn
        return RMSNormFn.apply(x)
    return ref.norm(x)


rms_norm = norm


def embed_norm(idx: torch.Tensor, wte: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if _cuda(wte) and dtype == torch.bfloat16 and wte.dtype == torch.float32:
        from .fused import EmbedNormFn
        return EmbedNormFn.apply(idx, wte)
    return ref.embed_norm(idx, wte, dtype)


def mix_norm(x, x0, resid_lambda, x0_lambda):
    """(xm, norm(xm)) with xm = resid_lambda * x + x0_lambda * x0."""
    if _cuda(x) and x.dtype == torch.bfloat16 and x0.dtype == torch.bfloat16:
        from .fused import MixNormFn
        return MixNormFn.apply(x, x0, resid_lambda, x0_lambda)
    return ref.mix_norm(x, x0, resid_lambda, x0_lambda)


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import LinearFn
        return LinearFn.apply(x, w, residual)
    return ref.linear(x, w, residual)


def linear_multi(x: torch.Tensor, ws: list[torch.Tensor]) -> torch.Tensor:
    """x @ cat(ws)^T as one GEMM (outputs concatenated on the last dim)."""
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import LinearMultiFn
        return LinearMultiFn.apply(x, *ws)
    return torch.cat([ref.linear(x, w) for w in ws], dim=-1)


def mlp_relu2(x, w_fc, w_proj, residual=None, tau: float = 0.0):
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import MLPRelu2Fn
        return MLPRelu2Fn.apply(x, w_fc, w_proj, residual, float(tau))
    return ref.mlp_relu2(x, w_fc, w_proj, residual, tau)


def rope_norm(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """norm(apply_rotary_emb(x)) for x [B, T, H, D]; cos/sin [1, T, 1, D/2]."""
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import RopeNormFn
        T = x.shape[1]
        c2 = cos.reshape(-1, cos.shape[-1])[:T].contiguous()
        s2 = sin.reshape(-1, sin.shape[-1])[:T].contiguous()
        return RopeNormFn.apply(x, c2, s2, 0)
    return ref.rope_norm(x, cos, sin)


def attention(q, k, v, causal: bool = True, scale: float | None = None, attn_mask=None):
    """q, k, v [B, T, H, D] -> [B, T, H, D].  CUDA: tcgen05 flash attention (causal or
    full, T % 128 == 0, head_dim 64 / 128); additive masks (document / sliding-window
    variants of the family) use the reference composition."""
    if _cuda(q) and q.dtype == torch.bfloat16 and attn_mask is None:
        from .flash_attention import FlashAttnFn, supported
        B, T, H, D = q.shape
        if supported(T, D):
            return FlashAttnFn.apply(q, k, v, causal, scale if scale is not None else D ** -0.5)
    return ref.attention(q, k, v, causal, scale, attn_mask)


def attention_qkv(qkv: torch.Tensor, cos, sin, n_head: int, head_dim: int, scale: float | None):
    """Plain-block attention core from the fused projection [B, T, 3C]:
    RoPE + QK-norm on q, k, then causal attention.  Returns [B, T, C]."""
    B, T, C3 = qkv.shape
    from .flash_attention import supported
    if _cuda(qkv) and qkv.dtype == torch.bfloat16 and supported(T, head_dim):
        from .fused import AttnQKVFn
        c2 = cos.reshape(-1, cos.shape[-1])[:T].contiguous()
        s2 = sin.reshape(-1, sin.shape[-1])[:T].contiguous()
        sc = scale if scale is not None else head_dim ** -0.5
        return AttnQKVFn.apply(qkv, c2, s2, B, T, n_head, head_dim, sc)
    Cd = C3 // 3
    q, k, v = qkv.split(Cd, dim=-1)
    q = ref.rope_norm(q.view(B, T, n_head, head_dim), cos, sin)
    k = ref.rope_norm(k.view(B, T, n_head, head_dim), cos, sin)
    y = ref.attention(q, k, v.view(B, T, n_head, head_dim), True, scale)
    return y.reshape(B, T, Cd)


def qkv_attention(x: torch.Tensor, ws: list[torch.Tensor], cos, sin, n_head: int, head_dim: int,
                  scale: float | None):
    """Plain-block attention from the block input x [B, T, C] and the q / k / v weights:
    projection, RoPE + QK-norm on q and k, causal attention.  Returns [B, T, C].  On CUDA
    with heads of 128 the RoPE + QK-norm runs in the projection GEMM's epilogue
    (``TFB_QKV_ROPE=0`` makes it a separate kernel after the projection)."""
    B, T, _ = x.shape
    if _cuda(x) and x.dtype == torch.bfloat16 and os.environ.get("TFB_QKV_ROPE", "1") != "0":
        from .fused import QKVRopeAttnFn, qkv_rope_supported
        if qkv_rope_supported(T, n_head, head_dim):
            c2 = cos.reshape(-1, cos.shape[-1])[:T].contiguous()
            s2 = sin.reshape(-1, sin.shape[-1])[:T].contiguous()
            sc = scale if scale is not None else head_dim ** -0.5
            return QKVRopeAttnFn.apply(x, c2, s2, B, T, n_head, head_dim, sc, *ws)
    return attention_qkv(linear_multi(x, ws), cos, sin, n_head, head_dim, scale)


def causal_conv(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv1d over time: x [B, T, C], w [C, 1, K]."""
    if _cuda(x) and x.dtype == torch.bfloat16 and w.dtype == torch.float32 and x.shape[-1] % 8 == 0 \
            and w.shape[-1] <= 8:
        from .fused import CausalConvFn
        return CausalConvFn.apply(x, w)
    return ref.causal_conv(x, w)


def ngram_lookup(idx: torch.Tensor, table: torch.Tensor, order: int, primes, mod: int, pad: int,
                 dtype: torch.dtype) -> torch.Tensor:
    """Rows of a hashed n-gram table for every position of idx [B, T] (see
    ``reference.ngram_rows``), cast to ``dtype``: [B, T, Dn].  On CUDA the hash and the
    gather are one kernel and the backward scatters into the fp32 table gradient."""
    if _cuda(table) and table.dtype == torch.float32 and dtype == torch.bfloat16 and table.shape[1] % 4 == 0:
        from .fused import NgramLookupFn
        return NgramLookupFn.apply(idx, table, int(order), tuple(int(p) for p in primes), int(mod), int(pad))
    return table[ref.ngram_rows(idx, order, primes, mod, pad)].to(dtype)


def lm_head_softcap_ce(x, w_lm, targets, softcap: float, vocab: int, reduction: str = "mean",
                       row_weight=None):
    """Fused lm_head GEMM + softcap + cross-entropy (+ its backward)."""
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import LMHeadSoftcapCEFn, softcap_ce_rows
        if reduction == "none":
            return softcap_ce_rows(x, w_lm, targets, softcap, vocab)
        return LMHeadSoftcapCEFn.apply(x, w_lm, targets, softcap, vocab, row_weight, reduction)
    logits = ref.linear(x, w_lm)[..., :vocab].float()
    return ref.softcap_cross_entropy(logits, targets, softcap, reduction,
                                     None if row_weight is None else row_weight.reshape(-1))


def softcap_logits(x, w_lm, softcap: float, vocab: int):
    if _cuda(x) and x.dtype == torch.bfloat16:
        from .fused import softcap_logits as f
        return f(x, w_lm, softcap, vocab)
    return ref.softcap_logits(x, w_lm, softcap, vocab)
