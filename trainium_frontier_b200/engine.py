"""Training engine: parameter / gradient layout, the optimizer step, DP gradient sync.

Memory layout (built once, after the optimizer groups are known):

* all trainable parameters live in ONE fp32 buffer and all gradients in ONE fp32
  buffer of the same layout (``param.data`` / ``param.grad`` are views), so
  zeroing, clipping, loss-scale checks and DP collectives are flat-buffer ops;
* the transformer blocks are cut into chunks of ``bucket_layers`` layers; inside a
  chunk the Muon matrices are ordered by shape group, so every (chunk, shape) run is
  one contiguous ``[K, rows, cols]`` stack -- Newton-Schulz reads it in place and the
  chunk is one gradient bucket that can be reduced as soon as backward leaves it;
* c_q / c_k / c_v of a block are adjacent, so the fused QKV GEMM reads one
  ``[3C, C]`` bf16 weight view and writes one ``[3C, C]`` fp32 gradient view;
* the bf16 copies of the Muon matrices (what the GEMMs read) are one buffer with the
  same layout, refreshed with a single cast after each optimizer step.

DP modes (``grad_sync``): ``per_param`` = the reference's per-tensor all_reduce after
backward (NCCL baseline); ``bucket`` = one all_reduce per chunk launched on a side
stream the moment backward finishes the chunk (overlapped); ``dist_muon`` = reduce-
scatter to owner ranks + owner-only Newton-Schulz + all-gather (parallel.dist_muon).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch.autograd import Function

from .config import RunConfig
from .optim.muon_adamw import MuonAdamW
from .runtime import world


@dataclass
class Bucket:
    index: int
    start: int          # element offset in the flat buffers
    end: int
    layers: tuple[int, ...]
    work: object = None
    ready: bool = False


class _GradReady(Function):
    """Identity in forward; its backward fires when every layer downstream of this
    point in the forward (i.e. the whole chunk) has produced its gradients."""

    @staticmethod
    def forward(ctx, x, engine, bucket_idx):
        ctx.engine = engine
        ctx.bucket_idx = bucket_idx
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        ctx.engine._on_bucket_ready(ctx.bucket_idx)
        return g, None, None


class ParamLayout:
    def __init__(self, model, optimizer: MuonAdamW, device: torch.device, bucket_layers: int = 4,
                 dist_world: int = 0, symm: bool = False):
        self.model = model
        self.device = device
        self.symm = symm
        blocks = list(model.transformer.h)
        L = len(blocks)
        self.bucket_layers = max(1, bucket_layers)
        self.dist_plans = None
        if dist_world > 1:
            self._build_dist(model, optimizer, device, dist_world)
            return
        layer_of: dict[int, int] = {}
        for i, b in enumerate(blocks):
            for p in b.parameters():
                layer_of[id(p)] = i
        muon_groups = [g for g in optimizer.param_groups if g["kind"] == "muon"]
        ordered: list[torch.nn.Parameter] = []
        seen: set[int] = set()
        chunk_ranges: list[tuple[int, int, tuple[int, ...]]] = []
        n_chunks = math.ceil(L / self.bucket_layers)
        for c in range(n_chunks):
            lay = tuple(range(c * self.bucket_layers, min(L, (c + 1) * self.bucket_layers)))
            start = len(ordered)
            for g in muon_groups:
                for p in g["params"]:
                    if layer_of.get(id(p)) in lay and id(p) not in seen:
                        ordered.append(p)
                        seen.add(id(p))
            # the block's non-Muon parameters (lambdas, gates) ride in the same chunk
            for li in lay:
                for p in blocks[li].parameters():
                    if p.requires_grad and id(p) not in seen:
                        ordered.append(p)
                        seen.add(id(p))
            chunk_ranges.append((start, len(ordered), lay))
        rest_start = len(ordered)
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                ordered.append(p)
                seen.add(id(p))
        frozen = [p for p in model.parameters() if not p.requires_grad]
        self.params = ordered
        self.offsets: dict[int, tuple[int, int]] = {}
        off = 0
        for p in ordered:
            n = p.numel()
            pad = (-off) % 4  # 16-byte alignment of every parameter (vector loads, TMA)
            off += pad
            self.offsets[id(p)] = (off, n)
            off += n
        self.total = off + ((-off) % 4)
        self.data = torch.zeros(self.total, dtype=torch.float32, device=device)
        self.grad = torch.zeros(self.total, dtype=torch.float32, device=device)
        with torch.no_grad():
            for p in ordered:
                o, n = self.offsets[id(p)]
                view = self.data[o:o + n].view(p.shape)
                view.copy_(p.detach().to(device=device, dtype=torch.float32))
                p.data = view
                p.grad = self.grad[o:o + n].view(p.shape)
            for p in frozen:
                p.data = p.data.to(device)
        for name, buf in list(model.named_buffers()):
            pass
        model.to(device)  # buffers (rotary tables, masks)
        # buckets: one per chunk + one for everything outside the blocks
        self.buckets: list[Bucket] = []
        for i, (s, e, lay) in enumerate(chunk_ranges):
            if e > s:
                bs = self.offsets[id(ordered[s])][0]
                last = ordered[e - 1]
                be = self.offsets[id(last)][0] + last.numel()
                self.buckets.append(Bucket(i, bs, be, lay))
        if rest_start < len(ordered):
            bs = self.offsets[id(ordered[rest_start])][0]
            self.buckets.append(Bucket(len(self.buckets), bs, self.total, ()))
        self.first_layer_bucket = {b.layers[0]: b.index for b in self.buckets if b.layers}
        # bf16 caches: one buffer for every 2-D parameter read by a GEMM
        self.mat_params = [p for p in ordered if p.dim() == 2 and p.shape[0] % 8 == 0 and p.shape[1] % 8 == 0]
        self._install_bf16_cache(model, device)

    def _place(self, ordered_offsets, total, model, device):
        """Allocate the flat buffers and re-point parameters at their offsets.  With
        ``symm`` the gradient buffer is a symmetric allocation peers can read."""
        self.total = total + ((-total) % 64)
        self.data = torch.zeros(self.total, dtype=torch.float32, device=device)
        self.grad_handle = None
        if self.symm:
            import torch.distributed._symmetric_memory as symm_mem
            self.grad = symm_mem.empty(self.total, dtype=torch.float32, device=device)
            self.grad.zero_()
            self.grad_handle = symm_mem.rendezvous(self.grad, dist.group.WORLD)
        else:
            self.grad = torch.zeros(self.total, dtype=torch.float32, device=device)
        self.offsets = {}
        frozen = [p for p in model.parameters() if not p.requires_grad]
        with torch.no_grad():
            for p, o in ordered_offsets:
                n = p.numel()
                self.offsets[id(p)] = (o, n)
                view = self.data[o:o + n].view(p.shape)
                view.copy_(p.detach().to(device=device, dtype=torch.float32))
                p.data = view
                p.grad = self.grad[o:o + n].view(p.shape)
            for p in frozen:
                p.data = p.data.to(device)
        model.to(device)

    def _build_dist(self, model, optimizer, device, world):
        """Rank-major layout of every bucket (see parallel.dist_muon)."""
        from .parallel.dist_muon import plan_buckets
        muon_ids = {id(p) for g in optimizer.param_groups if g["kind"] == "muon" for p in g["params"]}
        plans = plan_buckets(model, muon_ids, world, self.bucket_layers)
        placed: list[tuple[torch.nn.Parameter, int]] = []
        seen: set[int] = set()
        off = 0
        self.dist_bucket_range = []
        self.buckets = []
        for bi, plan in enumerate(plans):
            start = off
            for r in range(world):
                local = 0
                for u in plan.owners[r]:
                    for p in u.params:
                        placed.append((p, start + r * plan.seg_numel + local))
                        seen.add(id(p))
                        local += p.numel()
            off = start + world * plan.seg_numel
            self.dist_bucket_range.append((start, off))
            self.buckets.append(Bucket(bi, start, off, plan.layers))
        rest_start = off
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                off += (-off) % 4
                placed.append((p, off))
                seen.add(id(p))
                off += p.numel()
        off += (-off) % 64
        self.rest_range = (rest_start, off)
        self.buckets.append(Bucket(len(self.buckets), rest_start, off, ()))
        self.dist_plans = plans
        self._place(placed, off, model, device)
        self.params = [p for p, _ in placed]
        self.first_layer_bucket = {b.layers[0]: b.index for b in self.buckets if b.layers}
        self.mat_params = [p for p in self.params if p.dim() == 2 and p.shape[0] % 8 == 0 and p.shape[1] % 8 == 0]
        self._install_bf16_cache(model, device)

    def _install_bf16_cache(self, model, device):
        from .ops import fused
        lin_ids = set()
        for m in model.modules():
            if isinstance(m, torch.nn.Linear):
                lin_ids.add(id(m.weight))
        mats = [p for p in self.mat_params if id(p) in lin_ids]
        off = 0
        self.w16_offsets = {}
        for p in mats:
            off += (-off) % 8
            self.w16_offsets[id(p)] = (off, p.numel())
            off += p.numel()
        self.w16 = torch.empty(max(off, 8), dtype=torch.bfloat16, device=device) if device.type == "cuda" else None
        self.w16_params = mats if self.w16 is not None else []
        if self.w16 is None:
            return
        for p in mats:
            o, n = self.w16_offsets[id(p)]
            fused.set_w16(p, self.w16[o:o + n].view(p.shape))
        # fused QKV views: c_q, c_k, c_v adjacent in both the fp32 and bf16 buffers
        for blk in model.transformer.h:
            a = blk.attn
            ws = [a.c_q.weight, a.c_k.weight, a.c_v.weight]
            if not all(id(w) in self.w16_offsets for w in ws):
                continue
            o16 = [self.w16_offsets[id(w)][0] for w in ws]
            o32 = [self.offsets[id(w)][0] for w in ws]
            n = ws[0].numel()
            if all(ws[i].shape == ws[0].shape for i in range(3)) and o16[1] == o16[0] + n and o16[2] == o16[1] + n \
                    and o32[1] == o32[0] + n and o32[2] == o32[1] + n:
                rows = 3 * ws[0].shape[0]
                b16 = self.w16[o16[0]:o16[0] + 3 * n].view(rows, ws[0].shape[1])
                g32 = self.grad[o32[0]:o32[0] + 3 * n].view(rows, ws[0].shape[1])
                a.c_q.weight._tfb_fused = (b16, g32, tuple(id(w) for w in ws))
        self.refresh_bf16()

    @torch.no_grad()
    def refresh_bf16(self) -> None:
        """Re-cast every cached bf16 weight from its fp32 master (one fused pass per run
        of consecutive parameters)."""
        if self.w16 is None:
            return
        for p in self.w16_params:
            o, n = self.w16_offsets[id(p)]
            self.w16[o:o + n].copy_(self.data[self.offsets[id(p)][0]:self.offsets[id(p)][0] + n])
            p._tfb_w16_ver = p._version

    def zero_grad(self) -> None:
        self.grad.zero_()


class TrainEngine:
    """Owns model + optimizer + layout + loader and runs optimizer steps."""

    def __init__(self, model, optimizer: MuonAdamW, cfg: RunConfig, device: torch.device, grad_accum: int,
                 grad_sync: str = "auto"):
        self.model = model
        self.opt = optimizer
        self.cfg = cfg
        self.device = device
        self.grad_accum = grad_accum
        self.rank, self.world = world()
        if grad_sync == "auto":
            # the NVLink kernels over symmetric memory on GPUs, NCCL collectives elsewhere
            grad_sync = ("fused" if device.type == "cuda" else "dist_muon") if self.world > 1 else "none"
        if grad_sync == "fused" and (device.type != "cuda" or self.world < 2):
            grad_sync = "dist_muon" if self.world > 1 else "none"
        if self.world == 1:
            grad_sync = "none"
        self.grad_sync = grad_sync
        self.layout = ParamLayout(model, optimizer, device, cfg.bucket_layers,
                                  dist_world=self.world if grad_sync in ("dist_muon", "fused") else 0,
                                  symm=grad_sync == "fused")
        self.comm_stream = torch.cuda.Stream(device) if device.type == "cuda" else None
        self._sync_now = False
        self.clip_params = None
        self.dist_muon = None
        if grad_sync in ("dist_muon", "fused"):
            from .parallel.dist_muon import DistMuon
            self.dist_muon = DistMuon(self, optimizer, fused=grad_sync == "fused")
        self._install_markers()

    # ------------------------------------------------------------------ bucket hooks
    def _install_markers(self):
        engine = self
        for li, bidx in self.layout.first_layer_bucket.items():
            blk = self.model.transformer.h[li]
            if getattr(blk, "_tfb_marker_hook", None) is not None:
                blk._tfb_marker_hook.remove()

            def pre_hook(module, args, kwargs, _b=bidx):
                if not torch.is_grad_enabled() or engine.grad_sync not in ("bucket", "dist_muon", "fused"):
                    return None
                x = args[0]
                return (_GradReady.apply(x, engine, _b),) + tuple(args[1:]), kwargs

            blk._tfb_marker_hook = blk.register_forward_pre_hook(pre_hook, with_kwargs=True)

    def _on_bucket_ready(self, bidx: int) -> None:
        if not self._sync_now:
            return
        b = self.layout.buckets[bidx]
        if b.ready:
            return
        b.ready = True
        if self.grad_sync == "bucket" and self.cfg.clip_order == "global":
            self._launch_allreduce(b)
        elif self.grad_sync in ("dist_muon", "fused"):
            self.dist_muon.on_bucket_ready(b)

    def _launch_allreduce(self, b: Bucket) -> None:
        view = self.layout.grad[b.start:b.end]
        if self.comm_stream is not None:
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                b.work = dist.all_reduce(view, op=dist.ReduceOp.AVG, async_op=True)
        else:
            b.work = dist.all_reduce(view, op=dist.ReduceOp.AVG, async_op=True)

    def _finish_sync(self) -> None:
        if self.grad_sync == "per_param":
            from .parallel.ddp import sync_gradients
            sync_gradients(self.model)
            return
        if self.grad_sync == "bucket":
            for b in self.layout.buckets:
                if not b.ready or b.work is None:
                    self._launch_allreduce(b)
            for b in self.layout.buckets:
                if b.work is not None:
                    b.work.wait()
                    b.work = None
            if self.comm_stream is not None:
                torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        elif self.grad_sync in ("dist_muon", "fused"):
            self.dist_muon.finish_grad_sync()

    def _adamw_params(self):
        if not hasattr(self, "_adamw_cache"):
            self._adamw_cache = [p for g in self.opt.param_groups if g["kind"] in ("adamw", "rmsprop")
                                 for p in g["params"]]
        return self._adamw_cache

    # ------------------------------------------------------------------ step
    def clip_(self) -> torch.Tensor | None:
        if self.cfg.grad_clip <= 0:
            return None
        g = self.layout.grad
        total = torch.linalg.vector_norm(g)
        coef = torch.clamp(self.cfg.grad_clip / (total + 1e-6), max=1.0)
        g.mul_(coef)
        return total

    def forward_backward(self, batches, loss_scale: float = 1.0, zero_adamw: bool = True) -> torch.Tensor:
        """Runs the grad-accumulation micro-steps; returns the mean loss (device).

        ``zero_adamw=False`` keeps the AdamW / RMSProp gradients of the previous steps
        (AdamW updating every N steps, train.py:481-499): they keep accumulating until the
        step that applies them.  Averaging across ranks is linear, so re-averaging the
        accumulated sum every step equals the reference's deferred all-reduce."""
        if zero_adamw:
            self.layout.zero_grad()
        else:
            keep = [(p, p.grad.clone()) for p in self._adamw_params() if p.grad is not None]
            self.layout.zero_grad()
            for p, g in keep:
                p.grad.copy_(g)
        for b in self.layout.buckets:
            b.ready = False
            b.work = None
        inv = 1.0 / len(batches)
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        local_clip = self.cfg.clip_order == "local" and self.cfg.grad_clip > 0
        if self.dist_muon is not None:
            self.dist_muon.begin_step()
        ppc = getattr(self.model, "ppc", None)
        if ppc is not None:
            # pipeline: stages finish their buckets at different times, so the collectives
            # are issued after backward, in bucket order, on every rank
            from .parallel.pipeline import pipeline_forward_backward
            self._sync_now = False
            return pipeline_forward_backward(self.model, ppc, batches, loss_scale)
        for i, (x, y) in enumerate(batches):
            self._sync_now = (i == len(batches) - 1) and self.grad_sync in ("bucket", "dist_muon", "fused") \
                and not local_clip
            loss = self.model(x, y)
            (loss * (inv * loss_scale)).backward()
            total += loss.detach()
        self._sync_now = False
        return total * inv

    def sync_and_clip(self) -> torch.Tensor | None:
        norm = None
        if self.cfg.clip_order == "local" or self.grad_sync == "none":
            norm = self.clip_()
            self._finish_sync()
        else:
            self._finish_sync()
            if self.dist_muon is None:
                norm = self.clip_()
        return norm

    def optimizer_step(self, update_adamw: bool = True) -> None:
        if self.dist_muon is not None:
            self.dist_muon.step(update_adamw)
        else:
            self.opt.step(update_adamw)
        self.layout.refresh_bf16()
        tpc = getattr(self.model, "tpc", None)
        if tpc is not None:
            tpc.weights_version += 1
