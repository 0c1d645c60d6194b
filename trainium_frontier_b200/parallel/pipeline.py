"""Pipeline parallelism: the blocks are cut into ``pp`` contiguous stages, one per rank of a
pipeline group, and micro-batches flow through them over point-to-point sends
(``batch_isend_irecv``: one NCCL group of p2p sends / receives per boundary crossing on
GPUs, gloo on CPUs), GPipe order -- every micro-batch forward, then every backward in
reverse -- with the next activation's receive posted while the current micro-batch
computes.  The two tensors that cross a boundary together travel as one batch, which on
NCCL is also what keeps p2p traffic from being serialised as separate collectives.

What crosses a stage boundary is the residual stream ``x`` and the normed embedding
``x0`` that every block mixes in (``resid_lambda * x + x0_lambda * x0``); on the way
back, their gradients.  ``x0``'s gradient collects the contribution of every stage's
blocks as it travels back to the embedding on stage 0.

Parameters stay whole and replicated (the checkpoint is the single-device layout); a
stage computes with and writes gradients into only its own layers (stage 0 also the
embedding, the last stage the lm_head and final norm), so every other gradient is zero
there.  The last stage back-propagates ``pp * loss``: the data-parallel engine's average
over all ranks of the flat gradient buffer then equals the data-parallel mean of the full
gradient, and Muon / AdamW run unchanged on every rank.

The reference trains data parallel only (``train.py:4383-4528``); this is the optional
pipeline strategy of the build plan.
"""
from __future__ import annotations


import torch
import torch.distributed as dist


def stage_bounds(n_layer: int, pp: int, stage: int) -> tuple[int, int]:
    """[lo, hi) block range of a stage: contiguous, sizes differ by at most one."""
    base, rem = divmod(n_layer, pp)
    lo = stage * base + min(stage, rem)
    return lo, lo + base + (1 if stage < rem else 0)


class PipelineContext:
    """Pipeline groups over consecutive ranks: ranks [d * pp, (d + 1) * pp) form one pipeline
    (stage = rank % pp); ranks with equal stage form its data-parallel group."""

    def __init__(self, pp: int, n_layer: int):
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        if self.world % pp:
            raise ValueError(f"world {self.world} is not a multiple of pp={pp}")
        if n_layer < pp:
            raise ValueError(f"{n_layer} layers cannot fill {pp} pipeline stages")
        self.pp = pp
        self.stage = self.rank % pp
        self.first, self.last = self.stage == 0, self.stage == pp - 1
        self.prev = self.rank - 1 if not self.first else None
        self.next = self.rank + 1 if not self.last else None
        self.lo, self.hi = stage_bounds(n_layer, pp, self.stage)


def _send(ts: list[torch.Tensor], dst: int) -> list:
    """Send the tensors to ``dst`` as one batch; returns the requests."""
    return dist.batch_isend_irecv([dist.P2POp(dist.isend, t, dst) for t in ts])


def _recv(n: int, shape, dtype, device, src: int):
    """Post ``n`` receives from ``src`` as one batch; returns (buffers, requests)."""
    bufs = [torch.empty(shape, dtype=dtype, device=device) for _ in range(n)]
    return bufs, dist.batch_isend_irecv([dist.P2POp(dist.irecv, b, src) for b in bufs])


def _wait(reqs) -> None:
    for r in reqs:
        r.wait()


def pipeline_forward_backward(model, ppc: PipelineContext, batches, loss_scale: float = 1.0) -> torch.Tensor:
    """GPipe step over ``batches`` [(x, y), ...] (token ids on every stage; only stage 0
    reads x and only the last stage reads y).  Returns the mean loss on the last stage
    (zero elsewhere).  Gradients accumulate into the parameters' ``.grad``."""
    from .. import ops
    dev = model.get_device()
    dt = model.compute_dtype
    n = len(batches)
    inv = 1.0 / n
    blocks = list(model.transformer.h)[ppc.lo:ppc.hi]
    saved = []          # per micro-batch: (x_in, x0_in, x_out) on this stage, or the loss
    total = torch.zeros((), dtype=torch.float32, device=dev)
    B, T = batches[0][0].shape
    C = model.config.n_embd
    shape = (B, T, C)
    pending = []
    keep = []           # tensors with a send in flight stay referenced until it completes
    # ------------------------------------------------------------------ forward
    nxt = _recv(2, shape, dt, dev, ppc.prev) if not ppc.first else None
    for m, (x_ids, y_ids) in enumerate(batches):
        if ppc.first:
            x0 = ops.embed_norm(x_ids, model.transformer.wte.weight, dt)
            x = x0
            x_in = x0_in = None
        else:
            (xb, x0b), reqs = nxt
            _wait(reqs)
            if m + 1 < n:  # post the next receive while this micro-batch computes
                nxt = _recv(2, shape, dt, dev, ppc.prev)
            x_in = xb.requires_grad_(True)
            x0_in = x0b.requires_grad_(True)
            x, x0 = x_in, x0_in
        t = x.shape[1]
        cos, sin = model.cos[:, :t], model.sin[:, :t]
        for blk in blocks:
            x = blk(x, x0, None, cos, sin, None)
        if ppc.last:
            h = ops.norm(x)
            loss = ops.lm_head_softcap_ce(h, model.lm_head.weight, y_ids, model.rc.logit_softcap,
                                          model.config.vocab_size)
            total += loss.detach()
            saved.append((x_in, x0_in, loss))
        else:
            xs, x0s = x.detach(), x0.detach()
            keep += [xs, x0s]
            pending += _send([xs, x0s], ppc.next)
            saved.append((x_in, x0_in, (x, x0)))
    # ------------------------------------------------------------------ backward
    for m in reversed(range(n)):
        x_in, x0_in, out = saved[m]
        if ppc.last:
            (out * (inv * loss_scale * ppc.pp)).backward()
        else:
            (gx, gx0), reqs = _recv(2, shape, dt, dev, ppc.next)
            _wait(reqs)
            x_out, x0_out = out
            # Driven through the scalar <x_out, gx> (+ <x0, gx0> on the first stage): its
            # gradient with respect to x_out is exactly the received gx (the fp32 product's
            # backward casts gx back to bf16 without rounding), and the first backward node
            # is a plain PyTorch op, as in the single-device step.
            root = (x_out.float() * gx.float()).sum()
            if ppc.first:
                root = root + (x0_out.float() * gx0.float()).sum()
            root.backward()
            if not ppc.first:
                # x0 passes through this stage unchanged: add the gradient arriving from
                # the later stages to what this stage's blocks contributed
                x0_in.grad = gx0 if x0_in.grad is None else x0_in.grad + gx0
        if not ppc.first:
            gxi = x_in.grad if x_in.grad is not None else torch.zeros(shape, dtype=dt, device=dev)
            gx0i = x0_in.grad if x0_in.grad is not None else torch.zeros(shape, dtype=dt, device=dev)
            gxi, gx0i = gxi.contiguous(), gx0i.contiguous()
            keep += [gxi, gx0i]
            pending += _send([gxi, gx0i], ppc.prev)
        saved[m] = None
    _wait(pending)
    # every rank reports the step's mean loss (the last stages hold it; average over the
    # data-parallel pipelines)
    dist.all_reduce(total)
    return total * (inv * ppc.pp / ppc.world)
