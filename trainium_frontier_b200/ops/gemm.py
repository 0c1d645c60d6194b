"""Thin Python front-end of the tcgen05 GEMM (``csrc/kernels/gemm_sm100.cu``).

The three products of a linear layer read their operands in place:

* ``linear_fwd``  y[M,N]  = x[M,K] @ W[N,K]^T          A, B both K-major
* ``linear_dx``   dx[M,K] = dy[M,N] @ W[N,K]            B MN-major (W read as stored)
* ``linear_dw``   dW[N,K] (+)= dy[M,N]^T @ x[M,K]       A, B both MN-major, fp32 out,
                                                         split-K over the token axis
Fused epilogues: residual add, relu^2 (with the pre-activation kept for backward),
relu^2 backward, fp32 accumulate into the gradient buffer.

Reference counterpart: ``Linear.forward`` (``train.py:2237-2267``), which reaches cuBLAS
through ``F.linear`` on CUDA; the Newton-Schulz matmul chain (``train.py:3629-3636``).
"""
from __future__ import annotations

import math

import torch

from ._ext import C, err_word

EPI_BF16, EPI_RELU2, EPI_RELU2_BWD, EPI_F32 = 0, 1, 2, 3
_SMS: dict[int, int] = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def _bn(n: int) -> int:
    return 256 if (n % 256 == 0 or n > 256 and n % 256 > 128) else 128


def _split_k(tiles: int, kb_total: int, sms: int, max_split: int = 16, min_kb: int = 8) -> int:
    """Pick the K split that best fills whole waves of the persistent grid (wave
    quantization: 150 output tiles on 148 SMs would leave the second wave 1% full)."""
    best, best_eff = 1, tiles / (math.ceil(tiles / sms) * sms)
    if best_eff > 0.93:
        return 1
    for s in range(2, max_split + 1):
        if kb_total // s < min_kb:
            break
        n = tiles * s
        eff = n / (math.ceil(n / sms) * sms)
        if eff > best_eff + 0.03:
            best, best_eff = s, eff
    return best


def _gemm(a, a_mn, b, b_mn, M, N, K, out, epi, alpha=1.0, beta=0.0, R=None, D2=None, tau=0.0,
          split_k=1, bn=None, alpha_t=None, rcoef=1.0):
    C().gemm_bf16(a, a_mn, b, b_mn, M, N, K, out, epi, float(alpha), float(beta), R, D2, float(tau),
                  int(split_k), int(bn or _bn(N)), err_word(a.device), alpha_t, float(rcoef))
    return out


def _c2(t: torch.Tensor) -> torch.Tensor:
    """2-D view with a contiguous inner dimension (copy only if needed)."""
    if t.dim() != 2:
        t = t.reshape(-1, t.shape[-1])
    if t.stride(-1) != 1 or (t.stride(0) * t.element_size()) % 16 != 0 or t.data_ptr() % 16 != 0:
        t = t.contiguous()
    return t


def linear_fwd(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None, alpha: float = 1.0) -> torch.Tensor:
    x2, w2 = _c2(x), _c2(w)
    M, K = x2.shape
    N = w2.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    R = _c2(residual) if residual is not None else None
    return _gemm(x2, False, w2, False, M, N, K, out, EPI_BF16, alpha=alpha, R=R)


def linear_rope_fwd(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, T: int,
                    rope_cols: int, rstd: torch.Tensor | None = None) -> torch.Tensor:
    """x W^T (bf16) with RoPE + per-head RMSNorm (head_dim 128) applied in the GEMM epilogue
    to the first ``rope_cols`` output columns; position = row % T, cos / sin [>= T, 64].
    ``rstd`` (fp32, [rows * rope_cols / 128]) receives each head's reciprocal RMS."""
    x2, w2 = _c2(x), _c2(w)
    M = x2.shape[0]
    out = torch.empty((M, w2.shape[0]), dtype=torch.bfloat16, device=x.device)
    C().gemm_rope(x2, w2, out, cos, sin, int(T), int(rope_cols), rstd, err_word(x.device))
    return out


def linear_relu2_fwd(x: torch.Tensor, w: torch.Tensor, tau: float = 0.0):
    """(relu(x W^T - tau)^2, x W^T) in one pass; both bf16."""
    x2, w2 = _c2(x), _c2(w)
    M, K = x2.shape
    N = w2.shape[0]
    act = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    h = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _gemm(x2, False, w2, False, M, N, K, act, EPI_RELU2, D2=h, tau=tau)
    return act, h


def linear_dx(dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
              relu2_h: torch.Tensor | None = None, tau: float = 0.0, alpha_t=None,
              residual: torch.Tensor | None = None) -> torch.Tensor:
    """dx = dy @ W (+ residual); with ``relu2_h`` the result is multiplied by 2 relu(h - tau)."""
    dy2, w2 = _c2(dy), _c2(w)
    M, Nn = dy2.shape
    K = w2.shape[1]
    if out is None:
        out = torch.empty((M, K), dtype=torch.bfloat16, device=dy.device)
    if relu2_h is not None:
        return _gemm(dy2, False, w2, True, M, K, Nn, out, EPI_RELU2_BWD, R=_c2(relu2_h), tau=tau,
                     alpha_t=alpha_t)
    R = _c2(residual) if residual is not None else None
    return _gemm(dy2, False, w2, True, M, K, Nn, out, EPI_BF16, alpha_t=alpha_t, R=R)


def linear_decode(x: torch.Tensor, w: torch.Tensor, cache: dict, residual: torch.Tensor | None = None,
                  relu2: bool = False, tau: float = 0.0) -> torch.Tensor:
    """bf16 x @ W^T (+ residual | relu(. - tau)^2) for a few rows in ONE launch: split-K over
    the SMs into an fp32 workspace that the last split of each region converts and
    re-zeroes (``cache`` keeps one zeroed workspace + counter set per shape; safe inside
    CUDA graphs since nothing is allocated or memset per call)."""
    x2, w2 = _c2(x), _c2(w)
    M, K = x2.shape
    N = w2.shape[0]
    key = (M, N, K, x.device)
    if key not in cache:
        tiles = math.ceil(M / 128) * math.ceil(N / 128)
        cache[key] = (torch.zeros((M, N), dtype=torch.float32, device=x.device),
                      torch.zeros(tiles * 8, dtype=torch.int32, device=x.device),
                      max(2, min(math.ceil(K / 64), num_sms(x.device) // max(1, tiles))))
    ws, cnt, split = cache[key]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    C().gemm_splitk_fin(x2, w2, ws, cnt, out, None if residual is None else _c2(residual), bool(relu2),
                        float(tau), int(split), err_word(x.device))
    return out


def linear_dw(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor, accumulate: bool = True,
              alpha: float = 1.0, split_k: int | None = None, alpha_t=None) -> torch.Tensor:
    """out[N,K] (fp32) (+)= alpha * dy^T x."""
    dy2, x2 = _c2(dy), _c2(x)
    M, Nn = dy2.shape
    K = x2.shape[1]
    assert out.dtype == torch.float32 and out.shape == (Nn, K), (out.shape, (Nn, K))
    if split_k is None:
        bn = _bn(K)
        tiles = math.ceil(Nn / 128) * math.ceil(K / bn)
        split_k = _split_k(tiles, math.ceil(M / 64), num_sms(dy.device))
    return _gemm(dy2, True, x2, True, Nn, K, M, out, EPI_F32, alpha=alpha,
                 beta=1.0 if accumulate else 0.0, split_k=split_k, alpha_t=alpha_t)


def bmm_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, residual: torch.Tensor | None = None,
           alpha: float = 1.0, rcoef: float = 1.0) -> torch.Tensor:
    """Batched out[i] = alpha * a[i] @ b[i]^T (+ rcoef * residual[i]); a [B,M,K], b [B,N,K]."""
    Bt, M, K = a.shape
    N = b.shape[1]
    return _gemm(a, False, b, False, M, N, K, out, EPI_BF16, alpha=alpha, R=residual, rcoef=rcoef)


def bmm_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, residual: torch.Tensor | None = None,
           alpha: float = 1.0, rcoef: float = 1.0) -> torch.Tensor:
    """Batched out[i] = alpha * a[i] @ b[i] (+ rcoef * residual[i]); a [B,M,K], b [B,K,N]."""
    Bt, M, K = a.shape
    N = b.shape[2]
    return _gemm(a, False, b, True, M, N, K, out, EPI_BF16, alpha=alpha, R=residual, rcoef=rcoef)


def bmm_tn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, residual: torch.Tensor | None = None,
           alpha: float = 1.0, rcoef: float = 1.0) -> torch.Tensor:
    """Batched out[i] = alpha * a[i]^T @ b[i] (+ rcoef * residual[i]); a [B,K,M], b [B,K,N]."""
    Bt, K, M = a.shape
    N = b.shape[2]
    return _gemm(a, True, b, True, M, N, K, out, EPI_BF16, alpha=alpha, R=residual, rcoef=rcoef)


def matmul_f32out(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M,N] = a[M,K] @ b[N,K]^T in fp32 (used for fp32 logits)."""
    a2, b2 = _c2(a), _c2(b)
    M, K = a2.shape
    N = b2.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    return _gemm(a2, False, b2, False, M, N, K, out, EPI_F32)


def gemm_any(a: torch.Tensor, a_mn: bool, b: torch.Tensor, b_mn: bool, M: int, N: int, K: int,
             out: torch.Tensor, epi: int = EPI_BF16, **kw) -> torch.Tensor:
    return _gemm(a, a_mn, b, b_mn, M, N, K, out, epi, **kw)
