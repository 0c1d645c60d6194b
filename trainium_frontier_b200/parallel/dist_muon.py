"""Distributed Muon: each rank orthogonalises only the matrices it owns.

Per gradient bucket (a chunk of ``bucket_layers`` transformer blocks):

1. ownership: the chunk's Muon matrices are grouped into units (c_q/c_k/c_v of a block
   stay together so the fused QKV GEMM keeps reading one [3C, C] view; c_proj, c_fc and
   the MLP projection are units of one) and assigned largest-first (by Newton-Schulz
   cost) to the rank with the least cost accumulated over all buckets so far.  The flat buffers of the chunk are laid out rank-major -- rank 0's
   units, rank 1's units, ... each segment padded to the largest -- so
2. one ``reduce_scatter`` (AVG) of the chunk delivers to every rank the averaged
   gradient of exactly the matrices it owns; it is launched on a side stream the
   moment backward leaves the chunk (overlapped with the rest of backward);
3. the owner runs momentum / Nesterov / Newton-Schulz / NorMuon on its matrices and
   writes the final bf16 update ``g`` (what the reference subtracts after scaling); the
   fused path gathers the owner's matrices of every bucket into one stack per (group,
   shape) first, so the batched Newton-Schulz GEMMs stay large at 8 ranks;
4. one ``all_gather`` of the bf16 updates gives every rank every matrix's ``g``, and
   every rank applies ``w -= lr g + lr wd w [g w >= 0]`` itself (identical inputs ->
   identical fp32 masters on all ranks, at half the bytes of gathering fp32 weights).

Everything outside the blocks' Muon matrices (embeddings, lm_head, scalars, gates)
is all-reduced and updated with AdamW on every rank.  Gradient clipping uses the global
norm of the averaged gradient (owner partial sums of squares + the all-reduced rest,
one scalar all-reduce).

Reference counterparts: the per-rank ``_muon_step`` that runs Newton-Schulz on every
matrix (``train.py:4130-4336``) and the per-parameter ``all_reduce(AVG)`` of
``sync_gradients`` (``train.py:4412-4420``); the reference has no sharded Muon.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..config import POLAR_EXPRESS_COEFFS


@dataclass
class Unit:
    params: list          # parameters kept adjacent (same shape)
    numel: int


@dataclass
class BucketPlan:
    layers: tuple
    owners: list = field(default_factory=list)       # per rank: list[Unit]
    seg_numel: int = 0                                 # padded segment size (elements)


def unit_cost(u: Unit, steps: int = 5) -> float:
    """Estimated owner time of a unit (seconds on one B200): Newton-Schulz FLOPs at
    ~1 PFLOP/s plus ~40 bytes of elementwise traffic per element at ~6.5 TB/s.  An
    r x c matrix with n = min(r, c), m = max(r, c) costs 4 n^2 m + 2 n^3 per iteration
    (Gram product, its square, the product back), so a 1280 x 5120 matrix costs about
    three, not four, 1280 x 1280 ones -- owners are balanced on this, not on size."""
    r, c = u.params[0].shape[-2], u.params[0].shape[-1]
    n, m = min(r, c), max(r, c)
    flops = steps * (4.0 * n * n * m + 2.0 * n ** 3) * len(u.params)
    return flops / 1.0e15 + 40.0 * u.numel / 6.5e12


def plan_buckets(model, muon_param_ids: set[int], world: int, bucket_layers: int) -> list[BucketPlan]:
    blocks = list(model.transformer.h)
    L = len(blocks)
    plans = []
    # Newton-Schulz cost accumulated over the buckets: each unit goes to the rank with the
    # least total so far, so the owners' whole-step work is balanced (a per-bucket greedy
    # alone hands the heaviest unit of every bucket to the same rank)
    cum = [0.0] * world
    for c in range(math.ceil(L / bucket_layers)):
        lay = tuple(range(c * bucket_layers, min(L, (c + 1) * bucket_layers)))
        units: list[Unit] = []
        for li in lay:
            blk = blocks[li]
            a = blk.attn
            qkv = [a.c_q.weight, a.c_k.weight, a.c_v.weight]
            if all(id(w) in muon_param_ids for w in qkv) and all(w.shape == qkv[0].shape for w in qkv):
                units.append(Unit(qkv, sum(w.numel() for w in qkv)))
                taken = {id(w) for w in qkv}
            else:
                taken = set()
            for p in blk.parameters():
                if id(p) in muon_param_ids and id(p) not in taken:
                    units.append(Unit([p], p.numel()))
        cost = [0.0] * world
        loads = [0] * world
        owners: list[list[Unit]] = [[] for _ in range(world)]
        for u in sorted(units, key=lambda u: -unit_cost(u)):
            r = min(range(world), key=lambda i: (cum[i], cost[i], loads[i]))
            owners[r].append(u)
            cost[r] += unit_cost(u)
            cum[r] += unit_cost(u)
            loads[r] += u.numel
        # inside a rank: group by shape so each (rank, shape) run is one contiguous stack
        for r in range(world):
            owners[r].sort(key=lambda u: (tuple(u.params[0].shape), -len(u.params)))
        seg = max(loads) if loads else 0
        seg += (-seg) % 64
        plans.append(BucketPlan(lay, owners, seg))
    return plans


class DistMuon:
    """Owner-sharded Muon + DP sync for a TrainEngine whose layout follows ``plans``.

    ``fused=False``: NCCL reduce_scatter / all_gather (the baseline collectives).
    ``fused=True``:  the buffers are symmetric allocations and the collectives are this
    framework's own kernels over NVLink peer memory (``csrc/kernels/symm_sm100.cu``):
    a bounded device barrier per bucket, a P2P (or NVSwitch multimem) reduce-scatter
    that also produces the norm partial, a fused momentum / Nesterov / bf16 / Frobenius
    prologue, and a gather + apply kernel writing fp32 masters and bf16 caches."""

    def __init__(self, engine, optimizer, fused: bool = False):
        self.engine = engine
        self.opt = optimizer
        self.fused = fused
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        lay = engine.layout
        self.plans = lay.dist_plans
        dev = lay.grad.device
        self.device = dev
        # per-bucket receive (fp32 averaged owned grads) and gather (bf16 updates) buffers
        self.recv = [torch.zeros(p.seg_numel, dtype=torch.float32, device=dev) for p in self.plans]
        self.gath = [torch.zeros(p.seg_numel * self.world, dtype=torch.bfloat16, device=dev) for p in self.plans]
        self.works = [None] * len(self.plans)
        self.rest_work = None
        self.comm = engine.comm_stream
        # optimizer group of every Muon parameter
        self.group_of: dict[int, dict] = {}
        for g in optimizer.param_groups:
            if g["kind"] == "muon":
                for i, p in enumerate(g["params"]):
                    self.group_of[id(p)] = g
        # owner state: momentum / second moment per owned matrix
        self.state: dict[int, dict] = {}
        self.clip_coef = None
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        # optional phase timeline: a list that receives (name, CUDA event) pairs recorded on
        # the main stream at the phase boundaries of finish_grad_sync and step
        self.timeline = None
        self.goff = []
        off = 0
        for p in self.plans:
            self.goff.append(off)
            off += self.world * p.seg_numel
        if fused:
            self._init_symm(off)

    # ------------------------------------------------------------------ symmetric memory
    def _init_symm(self, upd_numel: int) -> None:
        import os
        import torch.distributed._symmetric_memory as symm_mem
        from ..ops._ext import C, err_word
        self.C = C()
        self.err = err_word(self.device)
        lay = self.engine.layout
        h = lay.grad_handle
        base = h.buffer_ptrs[self.rank]
        goff_bytes = lay.grad.data_ptr() - base
        self.grad_peers = [int(p) + goff_bytes for p in h.buffer_ptrs]
        self.pads = [int(p) for p in h.signal_pad_ptrs]
        use_nvls = os.environ.get("TFB_NVLS", "0") == "1" and os.environ.get("NCCL_NVLS_ENABLE", "1") != "0"
        mc = int(getattr(h, "multicast_ptr", 0) or 0)
        self.grad_mc = (mc + goff_bytes) if (use_nvls and mc) else 0
        self.upd = symm_mem.empty(max(upd_numel, 64), dtype=torch.bfloat16, device=self.device)
        self.upd.zero_()
        self.upd_handle = symm_mem.rendezvous(self.upd, dist.group.WORLD)
        ubase = self.upd_handle.buffer_ptrs[self.rank]
        uoff = self.upd.data_ptr() - ubase
        self.upd_peers = [int(p) + uoff for p in self.upd_handle.buffer_ptrs]
        self.epoch = 0
        self._runs_tables = {}
        torch.cuda.synchronize(self.device)
        dist.barrier()

    def _barrier(self) -> None:
        self.epoch += 1
        self.C.symm_barrier(self.pads, self.rank, self.epoch, self.err)

    def begin_step(self) -> None:
        self.sumsq.zero_()

    def mark(self, name: str) -> None:
        if self.timeline is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.timeline.append((name, e))

    # ------------------------------------------------------------------ grads
    def _bucket_view(self, b: int) -> torch.Tensor:
        s, e = self.engine.layout.dist_bucket_range[b]
        return self.engine.layout.grad[s:e]

    def on_bucket_ready(self, bucket) -> None:
        b = bucket.index
        if b >= len(self.plans):
            return
        self._launch_rs(b)

    def _launch_rs(self, b: int) -> None:
        if self.works[b] is not None:
            return
        if self.fused:
            s0, _ = self.engine.layout.dist_bucket_range[b]
            S = self.plans[b].seg_numel
            stream = self.comm if self.comm is not None else torch.cuda.current_stream(self.device)
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(stream):
                self._barrier()   # every rank has finished this bucket's backward
                self.C.symm_rs(self.grad_peers, s0 + self.rank * S, S, self.recv[b], 1.0 / self.world,
                               self.sumsq, self.grad_mc)
            self.works[b] = "fused"
            return
        src = self._bucket_view(b)
        if self.comm is not None:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                self.works[b] = dist.reduce_scatter_tensor(self.recv[b], src, op=dist.ReduceOp.AVG, async_op=True)
        else:
            self.works[b] = dist.reduce_scatter_tensor(self.recv[b], src, op=dist.ReduceOp.AVG, async_op=True)

    def finish_grad_sync(self) -> None:
        lay = self.engine.layout
        self.mark("sync:start")
        for b in range(len(self.plans)):
            self._launch_rs(b)
        rs, re_ = lay.rest_range
        rest = lay.grad[rs:re_]
        if self.comm is not None:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                self.rest_work = dist.all_reduce(rest, op=dist.ReduceOp.AVG, async_op=True)
        else:
            self.rest_work = dist.all_reduce(rest, op=dist.ReduceOp.AVG, async_op=True)
        for b in range(len(self.plans)):
            if self.works[b] != "fused":
                self.works[b].wait()
            self.works[b] = None
        self.rest_work.wait()
        self.rest_work = None
        if self.comm is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.comm)
        self.mark("sync:reduce-scatter tail + rest all-reduce")
        # global norm of the averaged gradient
        clip = self.engine.cfg.grad_clip
        self.clip_coef = None
        if clip > 0:
            if self.fused:
                sq = self.sumsq
            else:
                sq = torch.zeros(1, dtype=torch.float32, device=self.device)
                for b in range(len(self.plans)):
                    sq += self.recv[b].square().sum()
            sq_all = sq.clone()
            dist.all_reduce(sq_all, op=dist.ReduceOp.SUM)
            total = (sq_all + rest.square().sum()).sqrt()
            coef = torch.clamp(clip / (total + 1e-6), max=1.0)
            rest.mul_(coef)
            self.clip_coef = coef
        self.mark("sync:clip (norm all-reduce)")

    # ------------------------------------------------------------------ step
    def _owned_runs(self, b: int):
        """(shape, [params], offset in the rank segment) runs of this rank's matrices."""
        runs = []
        off = 0
        cur_shape, cur, cur_off = None, [], 0
        for u in self.plans[b].owners[self.rank]:
            for p in u.params:
                shp = tuple(p.shape)
                if shp != cur_shape:
                    if cur:
                        runs.append((cur_shape, cur, cur_off))
                    cur_shape, cur, cur_off = shp, [], off
                cur.append(p)
                off += p.numel()
        if cur:
            runs.append((cur_shape, cur, cur_off))
        return runs

    def _all_runs(self, b: int):
        """Per rank, (shape, [params], offset) runs -- for applying gathered updates."""
        out = []
        for r in range(self.world):
            off = 0
            cur_shape, cur, cur_off = None, [], 0
            runs = []
            for u in self.plans[b].owners[r]:
                for p in u.params:
                    shp = tuple(p.shape)
                    if shp != cur_shape:
                        if cur:
                            runs.append((cur_shape, cur, cur_off))
                        cur_shape, cur, cur_off = shp, [], off
                    cur.append(p)
                    off += p.numel()
            if cur:
                runs.append((cur_shape, cur, cur_off))
            out.append(runs)
        return out

    @torch.no_grad()
    def step(self, update_adamw: bool = True) -> None:
        if self.fused:
            return self._step_fused(update_adamw)
        from ..optim.muon_adamw import muon_direction
        lay = self.engine.layout
        opt = self.opt
        to_bf16 = lay.grad.is_cuda
        # AdamW / RMSProp groups: redundant on every rank (grads already averaged)
        for g in opt.param_groups:
            if g["kind"] == "adamw" and update_adamw:
                opt._adamw_step(g)
            elif g["kind"] == "rmsprop" and update_adamw:
                opt._rmsprop_step(g)
        works = []
        for b in range(len(self.plans)):
            seg = self.recv[b]
            upd = torch.zeros(self.plans[b].seg_numel, dtype=torch.bfloat16, device=self.device)
            for shape, params, off in self._owned_runs(b):
                K = len(params)
                n = K * params[0].numel()
                grp = self.group_of[id(params[0])]
                g = seg[off:off + n].view(K, *shape)
                if self.clip_coef is not None:
                    g = g * self.clip_coef
                w = torch.stack([p.detach() for p in params]) if not _adjacent(params) else _stack_view(params)
                st = self._state(params, grp)
                if to_bf16:
                    # the fused owner kernels (clip folded into the momentum prologue)
                    _fused_owner_direction(self, grp, seg[off:off + n].view(K, *shape), st,
                                           None if self.clip_coef is None else self.clip_coef.reshape(1),
                                           upd[off:off + n].view(K, *shape))
                    continue
                gq = muon_direction(opt, grp, w, g, st["mb"], st["second"], to_bf16)
                upd[off:off + n].copy_(gq.reshape(-1).to(torch.bfloat16))
            out = self.gath[b]
            if self.comm is not None:
                self.comm.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(self.comm):
                    works.append(dist.all_gather_into_tensor(out, upd, async_op=True))
                    upd.record_stream(self.comm)
            else:
                works.append(dist.all_gather_into_tensor(out, upd, async_op=True))
        for b in range(len(self.plans)):
            works[b].wait()
            if self.comm is not None:
                torch.cuda.current_stream(self.device).wait_stream(self.comm)
            S = self.plans[b].seg_numel
            for r, runs in enumerate(self._all_runs(b)):
                for shape, params, off in runs:
                    K = len(params)
                    n = K * params[0].numel()
                    grp = self.group_of[id(params[0])]
                    gq = self.gath[b][r * S + off:r * S + off + n].view(K, *shape)
                    w = _stack_view(params)
                    _apply_update(opt, grp, w, gq, params)

    def _state(self, params, grp):
        key = id(params[0])
        st = self.state.get(key)
        if st is None:
            K = len(params)
            shape = params[0].shape
            red_dim = -1 if shape[-2] >= shape[-1] else -2
            sshape = (K, shape[-2], 1) if red_dim == -1 else (K, 1, shape[-1])
            st = {"mb": torch.zeros(K, *shape, dtype=torch.float32, device=self.device),
                  "second": torch.zeros(sshape, dtype=torch.float32, device=self.device)}
            self.state[key] = st
        return st


def _adjacent(params) -> bool:
    from ..optim.muon_adamw import _stacked_view
    return _stacked_view(list(params)) is not None


def _stack_view(params):
    from ..optim.muon_adamw import _stacked_view
    v = _stacked_view(list(params))
    assert v is not None, "owned run is not contiguous"
    return v


def _apply_update(opt, grp, w, gq, params) -> None:
    """w -= lr g + lr wd w [g w >= 0]  (the reference's apply, lr cast to g's dtype)."""
    shape = params[0].shape
    ratio = max(1.0, shape[-2] / shape[-1]) ** 0.5
    lr_t, lrwd_t, _, _, _ = opt._muon_scalars(grp, params[0], ratio)
    if w.is_cuda:
        from ..ops.optim_kernels import muon_apply
        muon_apply(w, gq, lr_t, lrwd_t, params)
        return
    mask = (gq * w) >= 0
    w.sub_(lr_t.to(gq.dtype) * gq + lrwd_t * w * mask)


def _fused_owner_direction(dm, grp, g, st, coef, out):
    """Owner half on the GPU, written straight into this rank's update buffer ``out``:
    clip + momentum / Nesterov prologue, Frobenius normalisation, Newton-Schulz, NorMuon
    (``ops.optim_kernels.muon_owner_update``)."""
    from ..ops.optim_kernels import muon_owner_update, muon_stack_fusable
    from ..optim.muon_adamw import muon_direction
    opt = dm.opt
    shape = g.shape[1:]
    ratio = max(1.0, shape[-2] / shape[-1]) ** 0.5
    _lr, _lrwd, mom_t, one_mom_t, one_b2_t = opt._muon_scalars(grp, g, ratio)
    if not muon_stack_fusable(g, st["mb"], mom_t, _lr):
        # shapes the kernels do not take (e.g. a width not a multiple of 8): eager math
        gc = g * coef if coef is not None else g
        out.copy_(muon_direction(opt, grp, gc, gc, st["mb"], st["second"], True).to(out.dtype))
        return
    muon_owner_update(g, st["mb"], st["second"], mom_t, one_mom_t, one_b2_t,
                      min(grp["ns_steps"], len(POLAR_EXPRESS_COEFFS)), coef=coef, out=out)


def _owner_stacks(self):
    """This rank's matrices over ALL buckets, one stack per (param group, shape):
    [(group, shape, runs, K, grad stack, update stack, state)], built once.  The per-run
    momentum / second-moment states become views of one stack per (group, shape), so the
    owner math runs a few large batched Newton-Schulz GEMMs instead of several small ones
    per bucket (at 8 ranks an owner holds an eighth of each bucket, too little to fill
    the GPU)."""
    if getattr(self, "_stacks", None) is not None:
        return self._stacks
    by: dict = {}
    for b in range(len(self.plans)):
        for shape, params, off in self._owned_runs(b):
            grp = self.group_of[id(params[0])]
            by.setdefault((id(grp), shape), (grp, shape, []))[2].append((b, params, off, len(params)))
    stacks = []
    for grp, shape, runs in by.values():
        Kt = sum(r[3] for r in runs)
        red_dim = -1 if shape[-2] >= shape[-1] else -2
        sshape = (Kt, shape[-2], 1) if red_dim == -1 else (Kt, 1, shape[-1])
        mb = torch.zeros(Kt, *shape, dtype=torch.float32, device=self.device)
        second = torch.zeros(sshape, dtype=torch.float32, device=self.device)
        k = 0
        for _, params, _, K in runs:
            old = self.state.get(id(params[0]))
            if old is not None:  # e.g. restored from a checkpoint before the first step
                mb[k:k + K].copy_(old["mb"])
                second[k:k + K].copy_(old["second"])
            self.state[id(params[0])] = {"mb": mb[k:k + K], "second": second[k:k + K]}
            k += K
        gbuf = torch.empty(Kt, *shape, dtype=torch.float32, device=self.device)
        obuf = torch.empty(Kt, *shape, dtype=torch.bfloat16, device=self.device)
        stacks.append((grp, shape, runs, Kt, gbuf, obuf, {"mb": mb, "second": second}))
    self._stacks = stacks
    return stacks


def _step_fused(self, update_adamw: bool = True) -> None:
    """Owner math on whole-step stacks on the main stream (this rank's matrices of every
    bucket, gathered per (group, shape) from the reduce-scatter outputs), updates scattered
    into the symmetric update buffer, then one device barrier and one gather + apply
    launch over every bucket."""
    opt = self.opt
    self.mark("opt:start")
    for g in opt.param_groups:
        if g["kind"] == "adamw" and update_adamw:
            opt._adamw_step(g)
        elif g["kind"] == "rmsprop" and update_adamw:
            opt._rmsprop_step(g)
    self.mark("opt:adamw")
    # scalars of every group (lr*ratio, lr*ratio*wd, momentum, ...) staged once for the
    # owner kernels and the apply kernel
    for g in opt.param_groups:
        if g["kind"] == "muon":
            shape = g["params"][0].shape
            opt._muon_scalars(g, g["params"][0], max(1.0, shape[-2] / shape[-1]) ** 0.5)
    coef = self.clip_coef.reshape(1) if self.clip_coef is not None else None
    main = torch.cuda.current_stream(self.device)
    side = self.comm if self.comm is not None else main
    for grp, shape, runs, Kt, gbuf, obuf, st in self._owner_stacks():
        numel = shape[-2] * shape[-1]
        gflat, oflat = gbuf.view(-1), obuf.view(-1)
        k = 0
        for b, params, off, K in runs:
            gflat[k * numel:(k + K) * numel].copy_(self.recv[b][off:off + K * numel])
            k += K
        _fused_owner_direction(self, grp, gbuf, st, coef, obuf)
        k = 0
        for b, params, off, K in runs:
            base = self.goff[b] + self.rank * self.plans[b].seg_numel
            self.upd[base + off:base + off + K * numel].copy_(oflat[k * numel:(k + K) * numel])
            k += K
    self.mark("opt:owner Newton-Schulz + NorMuon")
    side.wait_stream(main)
    with torch.cuda.stream(side):
        self._barrier()  # every owner's updates are in its update buffer
        self.C.symm_ag_apply(self.upd_peers, self._runs_table_all())
    main.wait_stream(side)
    self.mark("opt:gather-apply")
    self._barrier()  # peers are done reading this rank's gradient and update buffers
    self.mark("opt:final barrier")


def _runs_table_all(self) -> torch.Tensor:
    tab = getattr(self, "_runs_all", None)
    if tab is None:
        tab = torch.cat([self._runs_table(b) for b in range(len(self.plans))], 0)
        self._runs_all = tab
    return tab


def _runs_table(self, b: int) -> torch.Tensor:
    tab = self._runs_tables.get(b)
    if tab is not None:
        return tab
    rows = []
    S = self.plans[b].seg_numel
    for r, runs in enumerate(self._all_runs(b)):
        for shape, params, off in runs:
            K = len(params)
            n = K * params[0].numel()
            grp = self.group_of[id(params[0])]
            dev_scalars = self.opt._scalar_cache[id(grp)]["muon"][1]
            w16 = getattr(params[0], "_tfb_w16", None)
            rows.append([r, self.goff[b] + r * S + off, params[0].data_ptr(),
                         w16.data_ptr() if w16 is not None else 0, n,
                         dev_scalars[0:1].data_ptr(), dev_scalars[1:2].data_ptr(), 0])
    tab = torch.tensor(rows, dtype=torch.int64)
    self._runs_tables[b] = tab
    return tab


DistMuon._step_fused = _step_fused
DistMuon._owner_stacks = _owner_stacks
DistMuon._runs_table = _runs_table
DistMuon._runs_table_all = _runs_table_all
