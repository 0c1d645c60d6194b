"""Roofline of the fused collectives against NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m trainium_frontier_b200.utils.comm_bench \
        [--what dp|tp] [--numel 393216000] [--rows 4] [--iters 10] [--json out.json]

``--what tp`` times the tensor-parallel GEMMs with the collective fused in (d26 shapes)
against NCCL all-gather / reduce-scatter plus the plain tcgen05 GEMM; roofline = max(FLOPs
at the measured sustained bf16 GEMM rate, NVLink bytes into this GPU at 770 GB/s).
The default (``dp``) is the data-parallel distributed-Muon pair:

Times, with CUDA events on the launching stream and the max over ranks:

* fused reduce-scatter (+ sum of squares): each rank reads its 1/N segment of the fp32
  gradient buffer from every peer over NVLink (``symm_rs``), against
  ``dist.reduce_scatter_tensor`` (AVG) on the same bytes;
* fused all-gather + apply: each rank reads every owner's bf16 update segment and applies it
  to the fp32 master and bf16 cache (``symm_ag_apply``), against
  ``dist.all_gather_into_tensor`` of the bf16 updates (which does no apply at all).

Roofline per path = max(bytes crossing NVLink into this GPU / link bandwidth, local HBM
bytes / HBM bandwidth), with the link bandwidth the measured 770 GB/s per direction peer
copy and the HBM bandwidth from the measured peaks file when present; the fraction
against NVLink 5's nominal 900 GB/s per direction is reported beside it.
The default size is the d20 model's Muon matrices (20 x (4 x 1280^2 + 2 x 1280 x 5120)).

Reference counterparts: its only gradient collectives, the per-parameter and flat-buffer
all-reduces (``train.py:4412-4460``).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0          # measured peer-copy bandwidth per direction on this B200 pool
LINK_GBS_NOMINAL = 900.0  # NVLink 5 per direction per GPU (context: fraction also reported against it)


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


def _gemm_peak() -> float:
    here = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(here, "..", "..", "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops_sustained", d.get("bf16_tflops", 1400.0)))
    except (OSError, ValueError):
        return 1400.0


def bench_tp(args) -> None:
    """Fused TP GEMMs at the d26 shapes (C 1664, 13 heads x 128 split 7/6, MLP 6656 split
    3328/3328, seq 4096, 4 sequences per rank) against NCCL collective + plain GEMM."""
    from ..ops import gemm
    from ..ops._ext import check_errors
    from ..parallel.tensor_parallel import EPI_RELU2, TPContext, tp_split
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    C, F, D, H = 1664, 6656, 128, 13
    Mr = args.rows * 4096
    tpc = TPContext(world, dev, Mr, C, 2)
    M = tpc.M
    _, nq = tp_split(H * D, world, rank, D)
    _, nf = tp_split(F, world, rank, 128)
    bf = torch.bfloat16
    x = torch.randn(Mr, C, device=dev).to(bf)
    wqkv = (torch.randn(3 * nq, C, device=dev) * 0.02).to(bf)
    wfc = (torch.randn(nf, C, device=dev) * 0.02).to(bf)
    wproj = (torch.randn(C, nq, device=dev) * 0.02).to(bf)
    wmp = (torch.randn(C, nf, device=dev) * 0.02).to(bf)
    y = torch.randn(M, nq, device=dev).to(bf)
    u = torch.randn(M, nf, device=dev).to(bf)
    res = torch.randn(Mr, C, device=dev).to(bf)
    h = torch.empty(M, nf, device=dev, dtype=bf)
    full = torch.empty(M, C, device=dev, dtype=bf)
    peak = _gemm_peak()
    out = {"world": world, "rows_per_rank": Mr, "gemm_peak_tflops": peak, "link_gbs": LINK_GBS}

    def ag(w, epi=0):
        def f():
            tpc.put_rows(0, x)
            tpc.ag_gemm(0, w, False, epi, D2=h if epi == EPI_RELU2 else None)
            tpc.put_rows(1, x)
            tpc.rs_gemm(y, wproj, False, res)   # keeps AG calls separated by an RS (buffer reuse rule)
        return f

    def nccl_ag(w, epi=0):
        def f():
            dist.all_gather_into_tensor(full, x)
            if epi == EPI_RELU2:
                gemm.linear_relu2_fwd(full, w)
            else:
                gemm.linear_fwd(full, w)
            z = gemm.linear_fwd(y, wproj)
            o = torch.empty(Mr, C, device=dev, dtype=bf)
            dist.reduce_scatter_tensor(o, z)
            o += res
        return f

    def rs(a, w):
        def f():
            tpc.rs_gemm(a, w, False, res)
        return f

    def nccl_rs(a, w):
        def f():
            z = gemm.linear_fwd(a, w)
            o = torch.empty(Mr, C, device=dev, dtype=bf)
            dist.reduce_scatter_tensor(o, z)
            o += res
        return f

    t_rs_proj = _time(rs(y, wproj), args.iters)
    t_rs_mlp = _time(rs(u, wmp), args.iters)
    n_rs_proj = _time(nccl_rs(y, wproj), args.iters)
    n_rs_mlp = _time(nccl_rs(u, wmp), args.iters)
    t_ag_qkv = _time(ag(wqkv), args.iters) - t_rs_proj
    t_ag_fc = _time(ag(wfc, EPI_RELU2), args.iters) - t_rs_proj
    n_ag_qkv = _time(nccl_ag(wqkv), args.iters) - n_rs_proj
    n_ag_fc = _time(nccl_ag(wfc, EPI_RELU2), args.iters) - n_rs_proj
    check_errors(dev)
    link_ag = (world - 1) * Mr * C * 2
    link_rs = (world - 1) * Mr * C * 2
    rows = {
        "ag_gemm_qkv": (t_ag_qkv, n_ag_qkv, 2.0 * M * C * 3 * nq, link_ag),
        "ag_gemm_fc_relu2": (t_ag_fc, n_ag_fc, 2.0 * M * C * nf, link_ag),
        "gemm_rs_attn_proj": (t_rs_proj, n_rs_proj, 2.0 * M * nq * C, link_rs),
        "gemm_rs_mlp_proj": (t_rs_mlp, n_rs_mlp, 2.0 * M * nf * C, link_rs),
    }
    for k, (t, tn, fl, link) in rows.items():
        roof = max(fl / (peak * 1e9), link / (LINK_GBS * 1e6))
        roof_nom = max(fl / (peak * 1e9), link / (LINK_GBS_NOMINAL * 1e6))
        out[k] = {"ms": t, "nccl_plus_gemm_ms": tn, "tflops": fl / t / 1e9, "roofline_ms": roof,
                  "frac_of_roofline": roof / t, "frac_of_roofline_nominal_900": roof_nom / t,
                  "nvlink_bytes_in": link}
    if rank == 0:
        print(json.dumps(out))
        if args.json:
            with open(args.json, "w") as f:
                json.dump(out, f, indent=1)
    tpc.close()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", default="dp", choices=["dp", "tp"])
    ap.add_argument("--numel", type=int, default=20 * (4 * 1280 * 1280 + 2 * 1280 * 5120))
    ap.add_argument("--rows", type=int, default=4, help="tp: sequences of 4096 tokens per rank")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--json", default="")
    args = ap.parse_args()
    if args.what == "tp":
        return bench_tp(args)
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
        roof_nom = max(link / (LINK_GBS_NOMINAL * 1e9), hbm / (peaks["hbm_gbs"] * 1e9)) * 1e3
        res[name] = {"ms": t, "roofline_ms": roof_ms, "frac_of_roofline": roof_ms / t,
                     "frac_of_roofline_nominal_900": roof_nom / t,
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
