"""MuonAdamW: Muon (Polar-Express Newton-Schulz + NorMuon second moment + sign-gated
weight decay) for the 2-D block matrices, AdamW for embeddings / lm_head / scalars /
gates, RMSProp for hashed n-gram tables.  Mirrors ``train.py:3522-4380``.

Numerics follow the reference op for op (``_muon_math``, ``train.py:3574-3647``):
momentum ``lerp`` then Nesterov ``lerp``; cast to the compute dtype; Frobenius
normalisation ``x / (||x|| * 1.01 + 1e-6)``; five Polar-Express iterations on the
smaller Gram side; NorMuon row/column second moment with renormalisation to the
pre-scale norm; update ``w -= lr*g + lr*wd*w*[g*w >= 0]`` with ``lr`` cast to g's dtype
before the multiply (the 0-dim promotion rule); ``lr`` scaled by
``max(1, rows/cols)^0.5`` in the logical orientation.  The scalars are staged exactly
as the reference stages them (lr*ratio in fp32, 1-momentum in fp64).

On the GPU the Newton-Schulz products are batched tcgen05 GEMMs with the polynomial
folded into the epilogues (``ops.newton_schulz``); on the CPU they are the reference's
own matmul chain.  When a group's parameters (and gradients) are laid out back to
back in one buffer -- the engine's layout -- the stacked ``[K, r, c]`` views are free
and no read-in / write-back copies are made.
"""
from __future__ import annotations

import torch

from ..config import POLAR_EXPRESS_COEFFS, RunConfig
from ..ops import newton_schulz as ns

ADAM_LIKE_KINDS = ("adamw", "rmsprop")


def _stacked_view(tensors: list[torch.Tensor]) -> torch.Tensor | None:
    """A [K, *shape] view if the tensors are consecutive equal-shape contiguous slices
    of one storage, else None."""
    if not tensors or any(t is None for t in tensors):
        return None
    t0 = tensors[0]
    if not t0.is_contiguous():
        return None
    n = t0.numel()
    base = t0.data_ptr()
    es = t0.element_size()
    for i, t in enumerate(tensors):
        if t.shape != t0.shape or not t.is_contiguous() or t.data_ptr() != base + i * n * es or t.dtype != t0.dtype:
            return None
    return torch.as_strided(t0, (len(tensors),) + tuple(t0.shape), (n,) + tuple(t0.stride()))


@torch.no_grad()
def _muon_math(w, g, mb, second, mom, one_mom, lr, lrwd, ns_steps: int, red_dim: int, one_beta2,
               to_bf16: bool, lr_fp32: bool) -> None:
    """Muon on one stack (in place on w, mb, second); the reference's op order."""
    mb.lerp_(g, one_mom)
    gn = torch.lerp(g, mb, mom)
    x = gn.bfloat16() if to_bf16 else gn
    x = x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)
    gq = ns.newton_schulz(x, ns_steps)
    v_mean = gq.float().square().mean(dim=red_dim, keepdim=True)
    red_size = gq.size(red_dim)
    v_norm = (v_mean.sum(dim=(-2, -1), keepdim=True) * red_size).sqrt()
    second.lerp_(v_mean, one_beta2)
    step_size = second.clamp_min(1e-10).rsqrt()
    scaled = (v_mean * red_size) * step_size.square()
    v_norm_new = scaled.sum(dim=(-2, -1), keepdim=True).sqrt()
    gq = gq * (step_size * (v_norm / v_norm_new.clamp_min(1e-10))).to(gq.dtype)
    mask = (gq * w) >= 0
    if lr.dim() > 0 and lr.dtype != gq.dtype:
        lr_g = lr.to(gq.dtype) * gq
    elif lr_fp32 and lr.dtype != gq.dtype:
        lr_g = lr * gq.float()
    else:
        lr_g = lr * gq
    w.sub_(lr_g + lrwd * w * mask)


@torch.no_grad()
def muon_direction(opt, group, w, g, mb, second, to_bf16: bool) -> torch.Tensor:
    """The Muon update direction of one stack (momentum, Nesterov, Newton-Schulz,
    NorMuon scaling) without applying it -- the owner's half of distributed Muon."""
    shape = w.shape[1:]
    red_dim = -1 if shape[-2] >= shape[-1] else -2
    ratio = max(1.0, shape[-2] / shape[-1]) ** 0.5
    _lr, _lrwd, mom_t, one_mom_t, one_b2_t = opt._muon_scalars(group, w, ratio)
    one_b2 = one_b2_t if group.get("beta2_tensor") else 1 - group["beta2"]
    ns_steps = min(group["ns_steps"], len(POLAR_EXPRESS_COEFFS))
    mb.lerp_(g, one_mom_t)
    gn = torch.lerp(g, mb, mom_t)
    x = gn.bfloat16() if to_bf16 else gn
    x = x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)
    gq = ns.newton_schulz(x, ns_steps)
    v_mean = gq.float().square().mean(dim=red_dim, keepdim=True)
    red_size = gq.size(red_dim)
    v_norm = (v_mean.sum(dim=(-2, -1), keepdim=True) * red_size).sqrt()
    second.lerp_(v_mean, one_b2)
    step_size = second.clamp_min(1e-10).rsqrt()
    scaled = (v_mean * red_size) * step_size.square()
    v_norm_new = scaled.sum(dim=(-2, -1), keepdim=True).sqrt()
    return gq * (step_size * (v_norm / v_norm_new.clamp_min(1e-10))).to(gq.dtype)


class MuonAdamW(torch.optim.Optimizer):
    def __init__(self, param_groups, muon_lr_fp32: bool = False, compute_dtype: torch.dtype | None = None):
        super().__init__(param_groups, defaults={})
        self.muon_lr_fp32 = muon_lr_fp32
        self.compute_dtype = compute_dtype
        self._scalar_cache: dict[int, dict] = {}

    # ------------------------------------------------------------------ scalars
    def _device_scalar(self, group, key: str, value: float, ref: torch.Tensor) -> torch.Tensor:
        cache = self._scalar_cache.setdefault(id(group), {})
        entry = cache.get(key)
        if entry is None:
            entry = (torch.empty((), dtype=torch.float32),
                     torch.zeros((), dtype=torch.float32, device=ref.device))
            cache[key] = entry
        host, dev = entry
        host.fill_(float(value))
        dev.copy_(host, non_blocking=False)
        return dev

    def _muon_scalars(self, group, ref: torch.Tensor, ratio: float):
        cache = self._scalar_cache.setdefault(id(group), {})
        entry = cache.get("muon")
        if entry is None:
            entry = (torch.empty(5, dtype=torch.float32),
                     torch.zeros(5, dtype=torch.float32, device=ref.device),
                     torch.empty((), dtype=torch.float32))
            cache["muon"] = entry
        host, dev, tmp = entry
        tmp.fill_(float(group["lr"]))
        tmp.mul_(ratio)
        host[0].fill_(float(tmp))
        tmp.mul_(float(group["weight_decay"]))
        host[1].fill_(float(tmp))
        mom = float(group["momentum"])
        host[2].fill_(mom)
        host[3].fill_(1.0 - mom)
        host[4].fill_(1.0 - float(group["beta2"]))
        dev.copy_(host)
        return dev[0], dev[1], dev[2], dev[3], dev[4]

    # ------------------------------------------------------------------ AdamW / RMSProp
    def _adamw_state(self, group):
        beta1, beta2 = group["betas"]
        params, grads, m, v, b1, b2 = [], [], [], [], [], []
        for p in group["params"]:
            if p.grad is None:
                continue
            st = self.state[p]
            if not st:
                st["step"] = 0
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] += 1
            params.append(p)
            grads.append(p.grad)
            m.append(st["exp_avg"])
            v.append(st["exp_avg_sq"])
            b1.append(1 - beta1 ** st["step"])
            b2.append(1 - beta2 ** st["step"])
        return params, grads, m, v, b1, b2

    @torch.no_grad()
    def _adamw_step(self, group):
        params, grads, exp_avgs, exp_avg_sqs, bias1, bias2 = self._adamw_state(group)
        if not params:
            return
        lr = self._device_scalar(group, "lr", group["lr"], params[0])
        beta1, beta2 = group["betas"]
        wd = group["weight_decay"]
        from ..ops import oracle_active
        if params[0].is_cuda and all(p.dtype == torch.float32 for p in params) and not oracle_active():
            from ..ops.optim_kernels import adamw_multi
            adamw_multi(params, grads, exp_avgs, exp_avg_sqs, lr, beta1, beta2, group["eps"], wd,
                        bias1, bias2, cautious=group.get("cautious_wd", False))
            return
        torch._foreach_lerp_(exp_avgs, grads, 1 - beta1)
        torch._foreach_lerp_(exp_avg_sqs, torch._foreach_mul(grads, grads), 1 - beta2)
        denom = torch._foreach_div(exp_avg_sqs, bias2)
        torch._foreach_sqrt_(denom)
        torch._foreach_add_(denom, group["eps"])
        update = torch._foreach_div(exp_avgs, bias1)
        torch._foreach_div_(update, denom)
        if wd != 0:
            if group.get("cautious_wd", False):
                for p, u in zip(params, update):
                    p.mul_(1 - lr * wd * ((u * p) > 0).to(p.dtype))
            else:
                torch._foreach_mul_(params, 1 - lr * wd)
        torch._foreach_mul_(update, lr)
        torch._foreach_sub_(params, update)

    @torch.no_grad()
    def _rmsprop_step(self, group):
        assert group["weight_decay"] == 0.0
        beta2 = group["betas"][1]
        params, grads, sqs, b2s = [], [], [], []
        for p in group["params"]:
            if p.grad is None:
                continue
            st = self.state[p]
            if not st:
                st["step"] = 0
                st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] += 1
            params.append(p)
            grads.append(p.grad.to(p.dtype))
            sqs.append(st["exp_avg_sq"])
            b2s.append(1 - beta2 ** st["step"])
        if not params:
            return
        lr = self._device_scalar(group, "lr", group["lr"], params[0])
        torch._foreach_lerp_(sqs, torch._foreach_mul(grads, grads), 1 - beta2)
        denom = torch._foreach_div(sqs, b2s)
        torch._foreach_sqrt_(denom)
        torch._foreach_add_(denom, group["eps"])
        update = torch._foreach_div(grads, denom)
        torch._foreach_mul_(update, lr.to(params[0].dtype) if params[0].dtype != torch.float32 else lr)
        torch._foreach_sub_(params, update)

    # ------------------------------------------------------------------ Muon
    def _muon_buffers(self, group):
        params = group["params"]
        p0 = params[0]
        state = self.state[p0]
        shape = p0.shape
        transposed = group.get("transposed", False)
        lshape = (shape[-1], shape[-2]) if transposed else shape
        red_dim = -1 if lshape[-2] >= lshape[-1] else -2
        if transposed:
            red_dim = -2 if red_dim == -1 else -1
        if "momentum_buffer" not in state:
            state["momentum_buffer"] = torch.zeros(len(params), *shape, dtype=p0.dtype, device=p0.device)
            sshape = (len(params), shape[-2], 1) if red_dim == -1 else (len(params), 1, shape[-1])
            state["second_momentum_buffer"] = torch.zeros(sshape, dtype=torch.float32, device=p0.device)
        return state, shape, lshape, red_dim

    @staticmethod
    def _runs(params) -> list[tuple[int, int]]:
        """Maximal runs of consecutive group members whose data AND grads are adjacent
        slices of one buffer (each run is processed as one in-place [K, r, c] stack)."""
        runs, i0 = [], 0
        for i in range(1, len(params) + 1):
            if i == len(params) or _stacked_view([params[i - 1], params[i]]) is None or \
                    _stacked_view([params[i - 1].grad, params[i].grad]) is None:
                runs.append((i0, i))
                i0 = i
        return runs

    @torch.no_grad()
    def _muon_step(self, group):
        params = group["params"]
        if not params:
            return
        p0 = params[0]
        state, shape, lshape, red_dim = self._muon_buffers(group)
        ratio = max(1.0, lshape[-2] / lshape[-1]) ** 0.5
        lr_t, lrwd_t, mom_t, one_mom_t, one_b2_t = self._muon_scalars(group, p0, ratio)
        depth = group.get("depth_mults")
        if depth is not None:
            lm = torch.tensor(depth[0], dtype=torch.float32, device=p0.device).view(-1, 1, 1)
            mm = torch.tensor(depth[1], dtype=torch.float32, device=p0.device).view(-1, 1, 1)
            one_mom_t = (one_mom_t.double() * mm.double()).float()
            mom_t = 1.0 - one_mom_t
            lr_t = lr_t * lm
            lrwd_t = lrwd_t * lm
        to_bf16 = (self.compute_dtype == torch.bfloat16) if self.compute_dtype is not None else p0.is_cuda
        ns_steps = min(group["ns_steps"], len(POLAR_EXPRESS_COEFFS))
        one_b2 = one_b2_t if group.get("beta2_tensor") else 1 - group["beta2"]
        all_have_grads = all(p.grad is not None for p in params)
        runs = self._runs(params) if all_have_grads else [(0, len(params))]
        for i0, i1 in runs:
            sub = params[i0:i1]
            g = _stacked_view([p.grad for p in sub]) if all_have_grads else None
            if g is None:
                g = torch.stack([p.grad if p.grad is not None else torch.zeros_like(p) for p in sub])
            w = _stacked_view(list(sub))
            inplace = w is not None
            if not inplace:
                w = torch.stack([p.detach() for p in sub])
            sl = slice(i0, i1)
            from ..ops import oracle_active
            if inplace and to_bf16 and not self.muon_lr_fp32 and torch.is_tensor(one_b2_t) and not oracle_active():
                from ..ops.optim_kernels import muon_owner_update, muon_stack_fusable
                mb_s = state["momentum_buffer"][sl]
                if muon_stack_fusable(g, mb_s, mom_t, lr_t) and w.dtype == torch.float32 and w.is_contiguous():
                    ob2 = one_b2 if torch.is_tensor(one_b2) else one_b2_t
                    muon_owner_update(g, mb_s, state["second_momentum_buffer"][sl], mom_t, one_mom_t, ob2,
                                      ns_steps, w=w, lr=lr_t, lrwd=lrwd_t)
                    continue
            _muon_math(w, g, state["momentum_buffer"][sl], state["second_momentum_buffer"][sl],
                       mom_t if mom_t.dim() == 0 else mom_t[sl], one_mom_t if one_mom_t.dim() == 0 else one_mom_t[sl],
                       lr_t if lr_t.dim() == 0 else lr_t[sl], lrwd_t if lrwd_t.dim() == 0 else lrwd_t[sl],
                       ns_steps, red_dim, one_b2, to_bf16, self.muon_lr_fp32)
            if not inplace:
                torch._foreach_copy_(sub, list(w.unbind(0)))

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def step(self, update_adamw: bool = True):
        for group in self.param_groups:
            kind = group["kind"]
            if kind == "adamw":
                if update_adamw:
                    self._adamw_step(group)
            elif kind == "rmsprop":
                if update_adamw:
                    self._rmsprop_step(group)
            elif kind == "muon":
                self._muon_step(group)
            else:
                raise ValueError(f"unknown optimizer kind: {kind}")

    @torch.no_grad()
    def zero_grad_selective(self, zero_adamw: bool = True) -> None:
        for group in self.param_groups:
            if group["kind"] in ADAM_LIKE_KINDS and not zero_adamw:
                continue
            for p in group["params"]:
                p.grad = None

    def adamw_param_ids(self) -> frozenset[int]:
        return frozenset(id(p) for g in self.param_groups if g["kind"] in ADAM_LIKE_KINDS for p in g["params"])


def setup_optimizer(model, cfg: RunConfig, compute_dtype: torch.dtype | None = None) -> MuonAdamW:
    """Parameter routing of ``GPT.setup_optimizer`` (train.py:3216-3410)."""
    from ..optim.schedules import muon_depth_mults
    scalar_params, matrix_params, local_conv_params, gate_params = [], [], [], []
    depth_of: dict[int, int] = {}
    for i, block in enumerate(model.transformer.h):
        for p in block.parameters():
            depth_of[id(p)] = i
        if block.local_conv is not None:
            local_conv_params.append(block.local_conv.weight)
        scalar_params.extend([block.resid_lambda, block.x0_lambda])
        if block.x0_gate_s is not None:
            scalar_params.append(block.x0_gate_s)
        if block.par_lambda_a is not None:
            scalar_params.extend([block.par_lambda_a, block.par_lambda_m])
        if block.scalar_gate is not None:
            matrix_params.append(block.scalar_gate.weight)
        if block.qk_shift_beta is not None and block.qk_shift_beta.requires_grad:
            gate_params.append(block.qk_shift_beta)
        if block.attn.head_gate is not None:
            gate_params.append(block.attn.head_gate_bias)
        matrix_params.extend(p for name, p in block.attn.named_parameters() if name != "head_gate_bias")
        matrix_params.extend(block.mlp.parameters())
    matrix_params.extend(p.weight for p in model.ngram_proj.values())
    engram_conv = []
    if getattr(model, "engram", None) is not None:
        matrix_params.extend(l.weight for l in (model.engram.w_k, model.engram.w_v, model.engram.w_q) if l is not None)
        if model.engram.conv is not None:
            engram_conv.append(model.engram.conv.weight)
    if model.out_pool_lambdas is not None:
        scalar_params.append(model.out_pool_lambdas)
    if model.out_bigram is not None:
        gate_params.extend([model.out_bigram_gate.weight, model.out_bigram_gate_bias])
    for p in scalar_params:
        if p.ndim > 1:
            raise ValueError(f"scalar group holds only scalars / 1-D vectors, got {tuple(p.shape)}")
    dscale = (model.config.n_embd / 768) ** -0.5
    groups = [
        dict(kind="adamw", params=list(model.transformer.wte.parameters()), lr=cfg.embedding_lr * dscale,
             betas=(cfg.embed_adamw_beta1, cfg.embed_adamw_beta2), eps=1e-10, weight_decay=cfg.embedding_wd),
        dict(kind="adamw", params=list(model.lm_head.parameters()), lr=cfg.unembedding_lr * dscale,
             betas=(cfg.embed_adamw_beta1, cfg.lm_head_beta2), eps=1e-10, weight_decay=cfg.lm_head_wd),
        dict(kind="adamw", params=scalar_params, lr=cfg.scalar_lr, betas=(cfg.scalar_beta1, cfg.scalar_beta2),
             eps=1e-10, weight_decay=0.0),
    ]
    if gate_params:
        groups.append(dict(kind="adamw", params=gate_params, lr=cfg.matrix_lr, betas=(0.9, 0.95), eps=1e-10,
                           weight_decay=0.0))
    ve_params = list(model.value_embeds.parameters())
    if ve_params:
        groups.append(dict(kind="adamw", params=ve_params, lr=cfg.embedding_lr * dscale,
                           betas=(cfg.embed_adamw_beta1, cfg.embed_adamw_beta2), eps=1e-10, weight_decay=cfg.ve_wd))
    ngram_params = list(model.ngram_embeds.parameters())
    if getattr(model, "engram", None) is not None:
        ngram_params.extend(model.engram.tables.parameters())
    if engram_conv:
        groups.append(dict(kind="adamw", params=engram_conv, lr=cfg.matrix_lr, betas=(0.9, 0.95), eps=1e-10,
                           weight_decay=0.0))
    if ngram_params:
        lr = (cfg.ngram_ve_lr if cfg.ngram_ve_lr > 0 else cfg.embedding_lr) * dscale
        rms = cfg.ngram_ve_opt == "rmsprop"
        groups.append(dict(kind="rmsprop" if rms else "adamw", params=ngram_params, lr=lr,
                           betas=(0.0, cfg.ngram_ve_beta2) if rms else (0.8, cfg.embed_adamw_beta2),
                           eps=1e-10, weight_decay=0.0, no_lr_decay=cfg.ngram_ve_flat_lr))
    if model.out_bigram is not None:
        groups.append(dict(kind="adamw", params=[model.out_bigram.weight],
                           lr=(cfg.out_bigram_lr if cfg.out_bigram_lr > 0 else cfg.unembedding_lr) * dscale,
                           betas=(0.8, 0.96), eps=1e-10, weight_decay=0.0))
    if local_conv_params and cfg.train_local_conv:
        groups.append(dict(kind="adamw", params=local_conv_params, lr=cfg.matrix_lr, betas=(0.9, 0.95),
                           eps=1e-10, weight_decay=0.0))
    depth_on = not (cfg.muon_depth_lr_bottom == 1.0 and cfg.muon_depth_lr_top == 1.0) or \
        (cfg.muon_depth_mom_bottom > 0.0 and cfg.muon_depth_mom_top > 0.0)
    for shape in sorted({tuple(p.shape) for p in matrix_params}):
        params = [p for p in matrix_params if tuple(p.shape) == shape]
        g = dict(kind="muon", params=params, lr=cfg.matrix_lr, momentum=0.95, beta2=cfg.muon_beta2,
                 ns_steps=cfg.muon_ns_steps, weight_decay=cfg.weight_decay, transposed=False)
        if depth_on:
            g["depth_mults"] = muon_depth_mults(cfg, [depth_of.get(id(p)) for p in params], model.config.n_layer)
        groups.append(g)
    for g in groups:
        if g["kind"] == "adamw" and cfg.cautious_wd:
            g["cautious_wd"] = True
    opt = MuonAdamW(groups, muon_lr_fp32=cfg.muon_lr_fp32, compute_dtype=compute_dtype)
    for group in opt.param_groups:
        group["initial_lr"] = group["lr"]
        if group.get("betas") is not None:
            group["initial_betas"] = tuple(group["betas"])
    return opt
