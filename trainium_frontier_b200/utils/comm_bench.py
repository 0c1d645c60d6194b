"""Roofline of the fused data-parallel collectives against NCCL, at the d20 Muon size.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m trainium_frontier_b200.utils.comm_bench \
        [--numel 393216000] [--iters 10] [--json out.json]

Times, with CUDA events on the launching stream and the max over ranks:

* fused reduce-scatter (+ sum of squares): each rank reads its 1/N segment of the fp32
  gradient buffer from every peer over NVLink (``symm_rs``), against
  ``dist.reduce_scatter_tensor`` (AVG) on the same bytes;
* fused all-gather + apply: each rank reads every owner's bf16 update segment and applies it
  to the fp32 master and bf16 cache (``symm_ag_apply``), against
  ``dist.all_gather_into_tensor`` of the bf16 updates (which does no apply at all).

Roofline per path = max(bytes crossing NVLink into this GPU / link bandwidth, local HBM
bytes / HBM bandwidth), with the link bandwidth the measured 770 GB/s per direction peer
copy (nominal 900) and the HBM bandwidth from the measured peaks file when present.
The default size is the d20 model's Muon matrices (20 x (4 x 1280^2 + 2 x 1280 x 5120)).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _peaks() -> dict:
    here = os.path.dirname(os.path.abspath(__file__))
    p = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d.get("hbm_gbs", 6650.0)), "source": "measured"}
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def _time(fn, iters: int, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--numel", type=int, default=20 * (4 * 1280 * 1280 + 2 * 1280 * 5120))
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--json", default="")
    args = ap.parse_args()
    import torch.distributed._symmetric_memory as symm_mem

    from ..ops._ext import C, check_errors, err_word
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    peaks = _peaks()
    n = (args.numel // (world * 4096)) * world * 4096
    seg = n // world
    grad = symm_mem.empty(n, dtype=torch.float32, device=dev)
    gh = symm_mem.rendezvous(grad, dist.group.WORLD)
    grad.normal_()
    gpeers = [int(p) for p in gh.buffer_ptrs]
    pads = [int(p) for p in gh.signal_pad_ptrs]
    upd = symm_mem.empty(seg, dtype=torch.bfloat16, device=dev)
    uh = symm_mem.rendezvous(upd, dist.group.WORLD)
    upd.normal_()
    upeers = [int(p) for p in uh.buffer_ptrs]
    out = torch.empty(seg, device=dev)
    sumsq = torch.zeros(1, device=dev)
    err = err_word(dev)
    epoch = [0]

    def barrier():
        epoch[0] += 1
        C().symm_barrier(pads, rank, epoch[0], err)

    def fused_rs():
        barrier()
        C().symm_rs(gpeers, rank * seg, seg, out, 1.0 / world, sumsq, 0)

    w = torch.randn(n, device=dev)
    w16 = w.to(torch.bfloat16)
    lr = torch.full((1,), 1e-3, device=dev)
    lrwd = torch.full((1,), 1e-5, device=dev)
    runs = torch.tensor([[r, 0, w.data_ptr() + r * seg * 4, w16.data_ptr() + r * seg * 2, seg,
                          lr.data_ptr(), lrwd.data_ptr(), 0] for r in range(world)], dtype=torch.int64)

    def fused_ag():
        barrier()
        C().symm_ag_apply(upeers, runs)

    rs_out = torch.empty(seg, device=dev)
    ag_out = torch.empty(n, dtype=torch.bfloat16, device=dev)
    plain_g = grad.clone()
    plain_u = upd.clone()
    res = {"world": world, "numel": n, "peaks": peaks, "link_gbs": LINK_GBS}
    t_rs = _time(fused_rs, args.iters)
    t_rs_nccl = _time(lambda: dist.reduce_scatter_tensor(rs_out, plain_g, op=dist.ReduceOp.AVG), args.iters)
    t_ag = _time(fused_ag, args.iters)
    t_ag_nccl = _time(lambda: dist.all_gather_into_tensor(ag_out, plain_u), args.iters)
    check_errors(dev)
    # roofline: NVLink bytes in, HBM bytes touched (per rank)
    rs_link = (world - 1) * seg * 4
    rs_hbm = world * seg * 4 + seg * 4            # every rank's segment is read once somewhere + output
    ag_link = (world - 1) * seg * 2
    ag_hbm = n * (4 + 4 + 2) + seg * 2            # master read+write, bf16 cache write, own update
    for name, t, link, hbm in (("fused_rs", t_rs, rs_link, rs_hbm), ("fused_ag_apply", t_ag, ag_link, ag_hbm)):
        roof_ms = max(link / (LINK_GBS * 1e9), hbm / (peaks["hbm_gbs"] * 1e9)) * 1e3
        res[name] = {"ms": t, "roofline_ms": roof_ms, "frac_of_roofline": roof_ms / t,
                     "nvlink_bytes_in": link, "hbm_bytes": hbm, "link_gbs_achieved": link / t / 1e6}
    res["nccl_reduce_scatter"] = {"ms": t_rs_nccl, "frac_of_roofline": res["fused_rs"]["roofline_ms"] / t_rs_nccl}
    res["nccl_all_gather_no_apply"] = {"ms": t_ag_nccl}
    if rank == 0:
        print(json.dumps(res))
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f, indent=1)
    del gh, uh
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
