"""One profiled optimizer step of a GPT config, for launch lists and kernel captures.

    python -m trainium_frontier_b200.utils.profile_step --preset d20 --rows 16 [--accum 1]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m trainium_frontier_b200.utils.profile_step \
        --preset d20 --rows 32 [--grad-sync fused]

Runs ``--warmup`` steps, then brackets exactly one step with cudaProfilerStart/Stop
(so ``ncu --profile-from-start off`` sees only that step) and NVTX ranges per phase.
Without a profiler attached it prints the per-phase CUDA-event times of that step; with
several ranks (distributed Muon) it also splits the sync and optimizer phases at the
distributed-Muon boundaries (reduce-scatter tail + rest all-reduce, clip, AdamW, owner
Newton-Schulz with the overlapped gather-apply, gather-apply tail, final barrier) and
reports every phase as the max over ranks.

Reference counterpart: ``research/scratch/phase_timer.py`` (per-phase synchronized
timing of a steady-state step).
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="d20")
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--accum", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--json", default="")
    ap.add_argument("--grad-sync", default="auto")
    args = ap.parse_args()
    import os
    import torch.distributed as dist
    from ..config import preset
    from ..optim.schedules import apply_schedules
    from ..train import Trainer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg0 = preset(args.preset)
    cfg = preset(args.preset, device_batch_size=args.rows, pack_factor=1, progress_mode="steps",
                 num_steps=10 ** 6, total_batch_size=args.rows * cfg0.seq_len * args.accum * world,
                 grad_sync=args.grad_sync, clip_order="global")
    tr = Trainer(cfg, dev, rank, world)
    batches = []
    for _ in range(tr.grad_accum):
        r = tr.loader.next().clone()
        batches.append((r[:, :-1], r[:, 1:]))
    ev = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for k in ("fwd_bwd", "sync_clip", "optimizer")}

    def step(profiled: bool):
        e = ev
        if profiled:
            torch.cuda.nvtx.range_push("fwd_bwd")
        e["fwd_bwd"][0].record()
        tr.engine.forward_backward(batches)
        e["fwd_bwd"][1].record()
        if profiled:
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push("sync_clip")
        e["sync_clip"][0].record()
        tr.engine.sync_and_clip()
        e["sync_clip"][1].record()
        if profiled:
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push("optimizer")
        apply_schedules(cfg, tr.opt, tr.step_idx, 0.0)
        e["optimizer"][0].record()
        tr.engine.optimizer_step()
        e["optimizer"][1].record()
        if profiled:
            torch.cuda.nvtx.range_pop()
        tr.step_idx += 1

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    dm = getattr(tr.engine, "dist_muon", None)
    if dm is not None:
        dm.timeline = []
    torch.cuda.cudart().cudaProfilerStart()
    step(True)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    out = {k: a.elapsed_time(b) for k, (a, b) in ev.items()}
    if dm is not None and dm.timeline:
        tl = dm.timeline
        for (_, e0), (name, e1) in zip(tl, tl[1:]):
            if not name.endswith(":start"):
                out[name] = e0.elapsed_time(e1)
        dm.timeline = None
    if world > 1:
        keys = sorted(out)
        t = torch.tensor([out[k] for k in keys], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out = {k: float(v) for k, v in zip(keys, t.tolist())}
        out["ranks"] = world
        out["reduction"] = "max over ranks"
    out["tokens"] = tr.tokens_per_step
    if rank == 0:
        print(json.dumps(out))
        if args.json:
            with open(args.json, "w") as f:
                json.dump(out, f, indent=1)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
