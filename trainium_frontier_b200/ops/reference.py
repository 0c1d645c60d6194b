"""fp32 PyTorch oracle of every fused op (the CPU path, and the numerics reference the
GPU tests compare the sm_100a kernels against).

Each function follows the reference's eager op order so a CPU run reproduces the
reference's CPU numerics: ``norm`` = parameter-free ``F.rms_norm`` (train.py:1432-1433),
``apply_rotary_emb`` half-split rotation (train.py:2415-2420), softcap
``S*tanh(z/S)`` then cross-entropy (train.py:2203-2215), relu^2 MLP (train.py:2218-2234).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def norm(x: torch.Tensor) -> torch.Tensor:
    return F.rms_norm(x, (x.size(-1),))


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    y1 = x1 * cos + x2 * sin
    y2 = x1 * (-sin) + x2 * cos
    return torch.cat((y1, y2), dim=-1)


def rope_norm(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return norm(apply_rotary_emb(x, cos, sin))


def embed_norm(idx: torch.Tensor, wte: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return norm(F.embedding(idx.long(), wte).to(dtype))


def mix_norm(x, x0, resid_lambda, x0_lambda):
    """xm = resid_lambda x + x0_lambda x0 in x's dtype (the shape-[1] fp32 lambdas are cast
    first, so a bf16 residual stream stays bf16 as in the fused kernel; for fp32 inputs this
    is the reference's expression unchanged)."""
    if resid_lambda.dtype != x.dtype:
        resid_lambda, x0_lambda = resid_lambda.to(x.dtype), x0_lambda.to(x.dtype)
    xm = resid_lambda * x + x0_lambda * x0
    return xm, norm(xm)


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    y = F.linear(x, w.to(x.dtype))
    return y if residual is None else residual + y


def relu_squared(h: torch.Tensor, tau: float = 0.0) -> torch.Tensor:
    if tau != 0.0:
        return F.relu(h - tau).square()
    return F.relu(h).square()


def mlp_relu2(x, w_fc, w_proj, residual=None, tau: float = 0.0):
    y = linear(relu_squared(linear(x, w_fc), tau), w_proj)
    return y if residual is None else residual + y


def attention(q, k, v, causal: bool = True, scale: float | None = None, attn_mask=None):
    """q/k/v as [B, T, H, D]; returns [B, T, H, D]."""
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if attn_mask is None:
        y = F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, scale=scale)
    else:
        y = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=attn_mask, scale=scale)
    return y.transpose(1, 2)


def causal_conv(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv1d over time of x [B, T, C] with w [C, 1, K] (K-1 zeros of left
    padding, the weight cast to x's dtype), train.py:1316-1329."""
    k = w.shape[-1]
    xt = F.pad(x.transpose(1, 2), (k - 1, 0))
    return F.conv1d(xt, w.to(x.dtype), groups=x.shape[-1]).transpose(1, 2)


def ngram_rows(idx: torch.Tensor, order: int, primes, mod: int, pad: int) -> torch.Tensor:
    """Hashed n-gram table rows of every position (train.py:3087-3140): the token and its
    one (bigram) or two (trigram) predecessors, each times a layer prime, XORed, modulo
    the table's prime row count; a missing predecessor is the pad id."""
    cur = idx.long()
    prev = F.pad(cur[:, :-1], (1, 0), value=pad)
    if order == 2:
        h = (prev * primes[0]) ^ (cur * primes[1])
    else:
        prev2 = F.pad(cur[:, :-2], (2, 0), value=pad)
        h = (prev2 * primes[0]) ^ (prev * primes[1]) ^ (cur * primes[2])
    return h % mod


def softcap_logits(x, w_lm, softcap: float, vocab_size: int):
    logits = F.linear(x, w_lm.to(x.dtype))[..., :vocab_size].float()
    return softcap * torch.tanh(logits / softcap)


def softcap_cross_entropy(logits, targets, softcap: float, reduction: str = "mean", weight=None,
                          ignore_index: int = -1):
    capped = softcap * torch.tanh(logits / softcap)
    loss = F.cross_entropy(capped.reshape(-1, capped.size(-1)), targets.reshape(-1).long(),
                           reduction="none" if (weight is not None or reduction == "none") else reduction,
                           ignore_index=ignore_index)
    if weight is not None and reduction == "mean":
        return (loss * weight).sum() / weight.sum()
    if reduction == "none":
        return loss.view(targets.shape)
    return loss
