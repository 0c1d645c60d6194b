"""Autograd wrappers of the sm_100a kernels (CUDA path of every op in ``ops``).

Weight gradients never go through autograd's AccumulateGrad: each linear's backward
accumulates ``dW`` straight into the fp32 ``param.grad`` buffer from the GEMM epilogue
(``linear_dw`` with beta = 1), and returns ``None`` for the parameter.  The bf16 copy
of each fp32 master weight that the GEMMs read is cached on the parameter and
re-cast only when the parameter's version counter moved (the optimizer's apply
kernel writes the cache directly, so in training it is never re-cast here).

The gradient of x0 (the normed embedding, an input of every block's residual mix) is
accumulated in fp32 across layers through a side buffer owned by the embedding node,
so 20+ bf16 partial sums are never rounded on the way.

Reference counterparts: relu² (``train.py:1465-1515``, eager ``train.py:2218-2234``),
RoPE + QK-norm forward / backward (``train.py:1543-1702``, wrapper ``train.py:2423-2436``),
softcapped cross-entropy (``train.py:1768-1925``, wrapper ``train.py:2163-2215``), the
bf16 weight cache of ``Linear`` (``train.py:2237-2267``), parameter-free RMSNorm
(``train.py:1432-1433``).
"""
from __future__ import annotations


import torch
from torch.autograd import Function

from . import gemm
from ._ext import C

BF16 = torch.bfloat16
_EMBED_DETERMINISTIC = __import__("os").environ.get("TFB_EMBED_GRAD_ATOMIC", "0") != "1"


# --------------------------------------------------------------------------- helpers
def w16(p: torch.Tensor) -> torch.Tensor:
    """bf16 view of a (fp32) weight, cached on the parameter object."""
    if p.dtype == BF16:
        return p.detach()
    cached = getattr(p, "_tfb_w16", None)
    if cached is not None and getattr(p, "_tfb_w16_ver", -1) == p._version:
        return cached
    if cached is not None and cached.shape == p.shape:
        cached.copy_(p.detach())
    else:
        cached = p.detach().to(BF16)
        p._tfb_w16 = cached
    p._tfb_w16_ver = p._version
    return cached


def set_w16(p: torch.Tensor, buf: torch.Tensor) -> None:
    """Install an externally managed bf16 cache (e.g. a view of a fused buffer)."""
    p._tfb_w16 = buf
    p._tfb_w16_ver = -1


def mark_w16_fresh(p: torch.Tensor) -> None:
    p._tfb_w16_ver = p._version


def grad_buf(p: torch.Tensor) -> torch.Tensor:
    """The fp32 gradient accumulator of a parameter (created zeroed on first use)."""
    if p.grad is None:
        p.grad = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
    return p.grad


def fused_group(ws: list[torch.Tensor]):
    """(bf16 [sum N, K], fp32 grad [sum N, K]) views covering the weights ``ws`` if an
    engine laid their caches and gradients out back to back, else None."""
    lead = ws[0]
    fg = getattr(lead, "_tfb_fused", None)
    if fg is None or fg[2] != tuple(id(w) for w in ws):
        return None
    buf16, gview, _ = fg
    if any(getattr(w, "_tfb_w16_ver", -1) != w._version for w in ws):
        for w, part in zip(ws, buf16.split([w.shape[0] for w in ws], 0)):
            part.copy_(w.detach())
            w._tfb_w16_ver = w._version
    return buf16, gview


def _2d(t):
    return t.reshape(-1, t.shape[-1])


# --------------------------------------------------------------------------- norms
class RMSNormFn(Function):
    @staticmethod
    def forward(ctx, x):
        x2 = _2d(x.contiguous())
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        C().rmsnorm_fwd(x2, y, rstd)
        ctx.save_for_backward(x2, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, rstd = ctx.saved_tensors
        dx = torch.empty_like(x2)
        C().rmsnorm_bwd(_2d(dy.contiguous()), x2, rstd, None, dx)
        return dx.view(ctx.shape)


class _X0Acc:
    __slots__ = ("buf", "started")

    def __init__(self):
        self.buf = None
        self.started = False


class EmbedNormFn(Function):
    @staticmethod
    def forward(ctx, idx, wte):
        B, T = idx.shape
        Cd = wte.shape[1]
        idx32 = idx if idx.dtype == torch.int32 else idx.to(torch.int32)
        out = torch.empty((B, T, Cd), dtype=BF16, device=wte.device)
        rstd = torch.empty(B * T, dtype=torch.float32, device=wte.device)
        C().embed_norm_fwd(idx32, wte.detach(), out, rstd)
        holder = _X0Acc()
        ctx.holder = holder
        ctx.wte = wte
        ctx.save_for_backward(idx32, rstd)
        out._tfb_x0acc = holder
        return out

    @staticmethod
    def backward(ctx, dout):
        idx32, rstd = ctx.saved_tensors
        holder = ctx.holder
        wte = ctx.wte
        gacc = holder.buf if holder.started else None
        gb = _2d(dout.contiguous()) if dout is not None else None
        if gacc is None and gb is None:
            return None, None
        if _EMBED_DETERMINISTIC and wte.shape[0] <= 8192 and wte.shape[1] <= 2048:
            # sorted segmented sums: the same bits every run (TFB_EMBED_GRAD_ATOMIC=1: the
            # one-pass scatter with fp32 atomics)
            C().embed_grad_det(idx32, wte.detach(), rstd, gacc, gb, grad_buf(wte))
        else:
            C().embed_norm_bwd(idx32, wte.detach(), rstd, gacc, gb, grad_buf(wte))
        holder.buf = None
        return None, None


class MixNormFn(Function):
    """xm = l_r * x + l_0 * x0 (bf16), h = norm(xm); returns (xm, h)."""

    @staticmethod
    def forward(ctx, x, x0, lam_r, lam_0):
        holder = getattr(x0, "_tfb_x0acc", None)
        x = x.contiguous()
        xm = torch.empty_like(x)
        h = torch.empty_like(x)
        M = x.numel() // x.shape[-1]
        rstd = torch.empty(M, dtype=torch.float32, device=x.device)
        C().mix_norm_fwd(x, x0, lam_r.detach(), lam_0.detach(), xm, h, rstd)
        ctx.holder = holder
        ctx.save_for_backward(x, x0, xm, rstd, lam_r, lam_0)
        return xm, h

    @staticmethod
    def backward(ctx, dxm, dh):
        x, x0, xm, rstd, lam_r, lam_0 = ctx.saved_tensors
        if dxm is None:
            dxm = torch.zeros_like(xm)
        if dh is None:
            dh = torch.zeros_like(xm)
        holder = ctx.holder
        own = holder is None
        if own:
            holder = _X0Acc()
        if holder.buf is None:
            holder.buf = torch.empty(x.shape, dtype=torch.float32, device=x.device)
            holder.started = False
        dx = torch.empty_like(x)
        dlr = torch.zeros(1, dtype=torch.float32, device=x.device)
        dl0 = torch.zeros(1, dtype=torch.float32, device=x.device)
        C().mix_norm_bwd(dxm.contiguous(), dh.contiguous(), x, x0, xm, rstd, lam_r.detach(), lam_0.detach(), dx,
                         holder.buf, not holder.started, dlr, dl0)
        holder.started = True
        dx0 = holder.buf.to(BF16) if own else None
        return dx, dx0, dlr.view_as(lam_r), dl0.view_as(lam_0)


# --------------------------------------------------------------------------- linears
class LinearFn(Function):
    """y = x W^T (+ residual).  W's gradient goes straight into W.grad (fp32)."""

    @staticmethod
    def forward(ctx, x, w, residual):
        x2 = gemm._c2(x)
        wb = w16(w)
        y = gemm.linear_fwd(x2, wb, residual=residual)
        ctx.save_for_backward(x2)
        ctx.w = w
        ctx.has_res = residual is not None
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], wb.shape[0])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        w = ctx.w
        wb = w16(w)
        dy2 = gemm._c2(dy)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm.linear_dx(dy2, wb).view(ctx.shape)
        if w.requires_grad:
            gemm.linear_dw(dy2, x2, grad_buf(w))
        return dx, None, (dy if ctx.has_res else None)


class LinearMultiFn(Function):
    """[y_1 | y_2 | ...] = x [W_1; W_2; ...]^T as one GEMM (fused QKV)."""

    @staticmethod
    def forward(ctx, x, *ws):
        x2 = gemm._c2(x)
        fg = fused_group(list(ws))
        if fg is not None:
            wb = fg[0]
        else:
            wb = torch.cat([w16(w) for w in ws], 0)
        y = gemm.linear_fwd(x2, wb)
        ctx.save_for_backward(x2)
        ctx.ws = ws
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], wb.shape[0])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        dx = _multi_backward(gemm._c2(dy), x2, list(ctx.ws), ctx.shape, ctx.needs_input_grad[0])
        return (dx,) + (None,) * len(ctx.ws)


class MLPRelu2Fn(Function):
    """residual + relu(x W_fc^T - tau)^2 W_proj^T, h kept for the backward."""

    @staticmethod
    def forward(ctx, x, w_fc, w_proj, residual, tau):
        x2 = gemm._c2(x)
        act, h = gemm.linear_relu2_fwd(x2, w16(w_fc), tau=tau)
        y = gemm.linear_fwd(act, w16(w_proj), residual=residual)
        ctx.save_for_backward(x2, act, h)
        ctx.w_fc, ctx.w_proj, ctx.tau = w_fc, w_proj, tau
        ctx.has_res = residual is not None
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        x2, act, h = ctx.saved_tensors
        dy2 = gemm._c2(dy)
        wp, wf = w16(ctx.w_proj), w16(ctx.w_fc)
        # dh = (dy W_proj) * 2 relu(h - tau)   (relu^2 backward fused in the epilogue)
        dh = gemm.linear_dx(dy2, wp, relu2_h=h, tau=ctx.tau)
        if ctx.w_proj.requires_grad:
            gemm.linear_dw(dy2, act, grad_buf(ctx.w_proj))
        dx = gemm.linear_dx(dh, wf).view(ctx.shape) if ctx.needs_input_grad[0] else None
        if ctx.w_fc.requires_grad:
            gemm.linear_dw(dh, x2, grad_buf(ctx.w_fc))
        return dx, None, None, (dy if ctx.has_res else None), None


# --------------------------------------------------------------------------- RoPE + QK norm
class RopeNormFn(Function):
    """norm(rope(x)) for x [B, T, H, D] (out of place)."""

    @staticmethod
    def forward(ctx, x, cos, sin, pos_offset=0):
        B, T, H, D = x.shape
        xc = x.contiguous()
        out = torch.empty_like(xc)
        rstd = torch.empty(B * T * H, dtype=torch.float32, device=x.device)
        C().rope_norm_fwd(xc.view(B * T, H * D), 0, H, D, cos, sin, T, pos_offset, rstd, out.view(B * T, H * D))
        ctx.save_for_backward(out, rstd, cos, sin)
        ctx.dims = (B, T, H, D)
        return out

    @staticmethod
    def backward(ctx, g):
        out, rstd, cos, sin = ctx.saved_tensors
        B, T, H, D = ctx.dims
        gx = g.contiguous().clone()
        C().rope_norm_bwd(gx.view(B * T, H * D), out.view(B * T, H * D), 0, H, D, cos, sin, T, rstd)
        return gx, None, None, None


class AttnQKVFn(Function):
    """Fused attention core of the plain block: RoPE + QK-norm of q and k from the
    [M, 3C] projection buffer, causal tcgen05 flash attention, output [B, T, C].
    The backward writes dq / dk / dv straight into one [M, 3C] gradient buffer and
    applies the RoPE + QK-norm backward in place on its q / k columns."""

    @staticmethod
    def forward(ctx, qkv, cos, sin, B, T, H, D, scale):
        from .flash_attention import flash_fwd
        Cd = H * D
        qkv2 = qkv.view(B * T, 3 * Cd)
        qkn = torch.empty((B * T, 2 * Cd), dtype=BF16, device=qkv.device)
        rstd = torch.empty(B * T * 2 * H, dtype=torch.float32, device=qkv.device)
        C().rope_norm_fwd(qkv2, 0, 2 * H, D, cos, sin, T, 0, rstd, qkn)
        o, lse = flash_fwd(qkn[:, :Cd], qkn[:, Cd:], qkv2[:, 2 * Cd:], B, T, H, D, scale, True)
        ctx.save_for_backward(qkv2, qkn, rstd, cos, sin, o, lse)
        ctx.meta = (B, T, H, D, scale)
        return o.view(B, T, Cd)

    @staticmethod
    def backward(ctx, dy):
        from .flash_attention import flash_bwd
        qkv2, qkn, rstd, cos, sin, o, lse = ctx.saved_tensors
        B, T, H, D, scale = ctx.meta
        Cd = H * D
        dqkv = torch.empty((B * T, 3 * Cd), dtype=BF16, device=dy.device)
        flash_bwd(qkn[:, :Cd], qkn[:, Cd:], qkv2[:, 2 * Cd:], o, dy.reshape(B * T, Cd), lse, B, T, H, D, scale,
                  True, dq=dqkv[:, :Cd], dk=dqkv[:, Cd:2 * Cd], dv=dqkv[:, 2 * Cd:])
        C().rope_norm_bwd(dqkv, qkn, 0, 2 * H, D, cos, sin, T, rstd)
        return dqkv.view(B, T, 3 * Cd), None, None, None, None, None, None, None


def _multi_backward(dy2, x2, ws, shape, need_dx):
    """dx = dy [W_1; W_2; ...] and each W_i's gradient accumulated into W_i.grad."""
    fg = fused_group(ws)
    if fg is not None:
        wb, gview = fg
        dx = gemm.linear_dx(dy2, wb).view(shape) if need_dx else None
        for w in ws:
            grad_buf(w)
        gemm.linear_dw(dy2, x2, gview)
        return dx
    wb = torch.cat([w16(w) for w in ws], 0)
    dx = gemm.linear_dx(dy2, wb).view(shape) if need_dx else None
    g = torch.zeros(wb.shape, dtype=torch.float32, device=dy2.device)
    gemm.linear_dw(dy2, x2, g, accumulate=False)
    for w, part in zip(ws, g.split([w.shape[0] for w in ws], 0)):
        if w.requires_grad:
            grad_buf(w).add_(part)
    return dx


def qkv_rope_supported(T: int, H: int, D: int) -> bool:
    """Shapes the projection-fused RoPE + QK-norm epilogue takes (heads of 128, whole
    128-row attention tiles)."""
    return D == 128 and T % 128 == 0


class QKVRopeAttnFn(Function):
    """Plain-block attention from the block input in two kernels: the fused [q | k | v]
    projection GEMM whose epilogue applies RoPE + QK-norm to the q and k heads (and writes
    their reciprocal RMS), then causal flash attention.  The normalised q / k overwrite
    their raw values, so no separate normalised copy is written or kept.

    Backward: flash attention backward into one [M, 3C] gradient buffer, the RoPE + QK-norm
    backward in place on its q / k columns, then dx and the three weight gradients."""

    @staticmethod
    def forward(ctx, x, cos, sin, B, T, H, D, scale, *ws):
        from .flash_attention import flash_fwd
        x2 = gemm._c2(x)
        fg = fused_group(list(ws))
        wb = fg[0] if fg is not None else torch.cat([w16(w) for w in ws], 0)
        Cd = H * D
        rstd = torch.empty(x2.shape[0] * 2 * H, dtype=torch.float32, device=x.device)
        qkv = gemm.linear_rope_fwd(x2, wb, cos, sin, T, 2 * Cd, rstd)
        o, lse = flash_fwd(qkv[:, :Cd], qkv[:, Cd:2 * Cd], qkv[:, 2 * Cd:], B, T, H, D, scale, True)
        ctx.save_for_backward(x2, qkv, rstd, cos, sin, o, lse)
        ctx.meta = (B, T, H, D, scale)
        ctx.ws = ws
        ctx.shape = x.shape
        return o.view(B, T, Cd)

    @staticmethod
    def backward(ctx, dy):
        from .flash_attention import flash_bwd
        x2, qkv, rstd, cos, sin, o, lse = ctx.saved_tensors
        B, T, H, D, scale = ctx.meta
        Cd = H * D
        dqkv = torch.empty((B * T, 3 * Cd), dtype=BF16, device=dy.device)
        flash_bwd(qkv[:, :Cd], qkv[:, Cd:2 * Cd], qkv[:, 2 * Cd:], o, dy.reshape(B * T, Cd), lse, B, T, H, D,
                  scale, True, dq=dqkv[:, :Cd], dk=dqkv[:, Cd:2 * Cd], dv=dqkv[:, 2 * Cd:])
        C().rope_norm_bwd(dqkv, qkv, 0, 2 * H, D, cos, sin, T, rstd)
        dx = _multi_backward(dqkv, x2, list(ctx.ws), ctx.shape, ctx.needs_input_grad[0])
        return (dx,) + (None,) * (7 + len(ctx.ws))


# --------------------------------------------------------------------------- lm_head + CE
def _lm_head_ce(x2, wb, targets, softcap: float, vocab: int, row_weight, write_dz: bool):
    """The lm_head GEMM with the softcap + cross-entropy statistics in its epilogue and one
    row pass after it (``gemm_ce``): returns the per-row losses and the [M, Vpad] bf16
    buffer holding dz (when ``write_dz``)."""
    M = x2.shape[0]
    Vp = wb.shape[0]
    tg = targets if targets.dim() == 2 else targets.view(1, -1)
    if tg.stride(-1) != 1:
        tg = tg.contiguous()
    dz = torch.empty((M, Vp), dtype=BF16, device=x2.device)
    tiles_n = (Vp + 255) // 256
    part = torch.empty(M * 2 * tiles_n, dtype=torch.float32, device=x2.device)
    yc = torch.empty(M, dtype=torch.float32, device=x2.device)
    loss_rows = torch.empty(M, dtype=torch.float32, device=x2.device)
    rw = None if row_weight is None else row_weight.reshape(-1).float().contiguous()
    C().gemm_ce(x2, wb, dz, tg, tg.shape[1], rw, int(vocab), float(softcap), part, yc, loss_rows,
                bool(write_dz), gemm.err_word(x2.device))
    return loss_rows, dz, tg


def _ce_fusable(x2, wb) -> bool:
    """The CE statistics ride in the lm_head GEMM's epilogue (TFB_CE_FUSED=0: the GEMM
    stores logits and the two-pass row kernel computes the loss and dlogits)."""
    import os
    return wb.shape[0] % 256 == 0 and x2.shape[1] % 8 == 0 and os.environ.get("TFB_CE_FUSED", "1") != "0"


class LMHeadSoftcapCEFn(Function):
    """loss = CE(S tanh(x W^T / S)[:, :V], targets), forward and dlogits in one GEMM.

    The lm_head GEMM's epilogue computes the softcap, the per-row partial sums of the
    softmax denominator and the target logit while it stores the bf16 logits; one row
    pass then writes the losses and turns the logits into dlogits in place (one read and
    one write of the [tokens, vocab] buffer instead of the former two reads and a write).
    ``row_weight`` (fp32 per token, or None) gives the byte-weighted mean; targets < 0
    are ignored.  The upstream gradient scalar is applied on the device inside the two
    backward GEMMs."""

    @staticmethod
    def forward(ctx, x, w, targets, softcap, vocab, row_weight, reduction):
        x2 = gemm._c2(x)
        wb = w16(w)
        M = x2.shape[0]
        if _ce_fusable(x2, wb):
            loss_rows, dz, tg = _lm_head_ce(x2, wb, targets, softcap, vocab, row_weight, True)
        else:
            dz = gemm.linear_fwd(x2, wb)
            loss_rows = torch.empty(M, dtype=torch.float32, device=x.device)
            tg = targets if targets.dim() == 2 else targets.view(1, -1)
            if tg.stride(1) != 1:
                tg = tg.contiguous()
            C().softcap_ce(dz, tg, tg.shape[1], row_weight, vocab, float(softcap), 1.0, loss_rows, True)
        if row_weight is not None:
            denom = (row_weight.reshape(-1) * (tg.reshape(-1) >= 0)).sum()
        else:
            denom = (tg >= 0).sum().to(torch.float32)
        inv = 1.0 / denom.clamp_min(1.0)
        loss = loss_rows.sum() * inv
        ctx.save_for_backward(x2, dz, inv)
        ctx.w = w
        ctx.shape = x.shape
        return loss

    @staticmethod
    def backward(ctx, g):
        x2, dz, inv = ctx.saved_tensors
        w = ctx.w
        alpha_t = (g.float() * inv).reshape(1).contiguous()
        wb = w16(w)
        dx = gemm.linear_dx(dz, wb, alpha_t=alpha_t).view(ctx.shape)
        if w.requires_grad:
            gemm.linear_dw(dz, x2, grad_buf(w), alpha_t=alpha_t)
        return dx, None, None, None, None, None, None


def softcap_logits(x, w, softcap: float, vocab: int) -> torch.Tensor:
    """Inference/eval logits: S tanh(z / S) of the bf16 lm_head product, fp32 [.., V]."""
    x2 = gemm._c2(x)
    z = gemm.linear_fwd(x2, w16(w))[:, :vocab].float()
    z = softcap * torch.tanh(z / softcap)
    return z.view(*x.shape[:-1], vocab)


def softcap_ce_rows(x, w, targets, softcap: float, vocab: int) -> torch.Tensor:
    """Per-token softcapped CE (no gradient), 0 where target < 0: the lm_head GEMM with the
    CE epilogue in its statistics-only form (no logits are stored)."""
    x2 = gemm._c2(x)
    wb = w16(w)
    if _ce_fusable(x2, wb):
        loss_rows, _dz, _tg = _lm_head_ce(x2, wb, targets, softcap, vocab, None, False)
        return loss_rows.view(targets.shape)
    logits = gemm.linear_fwd(x2, wb)
    loss_rows = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
    tg = targets if targets.dim() == 2 else targets.view(1, -1)
    C().softcap_ce(logits, tg.contiguous(), tg.shape[1], None, vocab, float(softcap), 1.0, loss_rows, False)
    return loss_rows.view(targets.shape)


# --------------------------------------------------------------------------- conv / n-gram
class CausalConvFn(Function):
    """Depthwise causal conv1d (x bf16 [B, T, C], w fp32 [C, 1, K]); the weight gradient is
    reduced deterministically and added straight into ``w``'s fp32 gradient buffer."""

    @staticmethod
    def forward(ctx, x, w):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        C().causal_conv_fwd(xc, w.detach(), y)
        ctx.save_for_backward(xc)
        ctx.w = w
        return y

    @staticmethod
    def backward(ctx, dy):
        (xc,) = ctx.saved_tensors
        w = ctx.w
        B, T, Cc = xc.shape
        K = w.shape[-1]
        dx = torch.empty_like(xc)
        runs = B * ((T + 63) // 64)
        part = torch.empty(runs * Cc * K, dtype=torch.float32, device=xc.device)
        C().causal_conv_bwd(xc, w.detach(), dy.contiguous(), dx, grad_buf(w).view(-1), part, True)
        return dx, None


class NgramLookupFn(Function):
    """Hashed n-gram row ids computed and the fp32 rows gathered (bf16 out) in one kernel;
    the backward adds every position's gradient row into the table's fp32 gradient."""

    @staticmethod
    def forward(ctx, idx, table, order, primes, mod, pad):
        B, T = idx.shape
        Dn = table.shape[1]
        idx32 = idx.to(torch.int32).contiguous()
        out = torch.empty((B, T, Dn), dtype=BF16, device=table.device)
        rows = torch.empty((B, T), dtype=torch.int32, device=table.device)
        p = tuple(primes) + (0,) * (3 - len(primes))
        C().ngram_gather(idx32, order, p[0], p[1], p[2], mod, pad, table.detach(), out, rows)
        ctx.save_for_backward(rows)
        ctx.table = table
        return out

    @staticmethod
    def backward(ctx, dout):
        (rows,) = ctx.saved_tensors
        C().ngram_scatter(rows, dout.contiguous(), grad_buf(ctx.table))
        return None, None, None, None, None, None
