"""Headline benchmark: d20 GPT pretraining throughput (tokens/s, max over ranks).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: 20 layers, d_model 1280, 10 heads x 128, relu^2 MLP 5120, vocab 8192, seq 2048,
global batch 524,288 tokens (fixed as N grows -> strong scaling), bf16 compute, fp32
master weights, MuonAdamW; random-init weights and a seeded synthetic Zipf token
stream.  Every timed step is a full optimizer step (all micro-steps, gradient sync,
clip, schedules, optimizer, bf16 weight refresh).

Two numbers are reported:
* ``value``: device time of K steps with inputs already resident (CUDA events on the
  launching stream, barrier + synchronize on both sides, max over ranks);
* ``e2e.value``: the same K steps through the public API ``Trainer.train_step()``,
  which per step copies that step's token rows host->device from pinned memory and
  reads the loss back device->host (wall clock around the loop, max over ranks).
Activations per micro-step are several GB, far above the 126 MB L2, so no explicit
flush is needed between steps.

``--impl library`` is a separately labelled comparator, not the reference: this
framework's model, engine and optimizer with every op routed through its PyTorch oracle
(bf16 cuBLAS GEMMs, SDPA attention, eager elementwise / optimizer math) -- how the same
model fares on library kernels.

``--impl reference`` runs the unmodified reference (``baseline/_ref/train.py``,
installed from the reference tree) through its own module API and stock code path
(torch.compile/inductor, SDPA, its eager Muon, per-parameter all-reduce) on the same
shape, with the same synthetic token stream, and prints the same JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PUBLISHED_TOKS = None  # the reference publishes no B200 number for this config
METRIC = "train tok/s (max over ranks) at 1/2/4/8 B200; step ms; held-out bpb at fixed budget"
CONFIGS = {
    "d20": {"model": "d20 GPT (20L, d1280, 10x128 heads, relu2 MLP 5120, vocab 8192)",
            "global_batch": 524288, "seq_len": 2048},
    "d12": {"model": "d12 GPT (12L, d768, 6x128 heads, relu2 MLP 3072, vocab 8192)",
            "global_batch": 524288, "seq_len": 2048},
    "d26": {"model": "d26 GPT (26L, d1664, 13x128 heads, relu2 MLP 6656, vocab 8192)",
            "global_batch": 1048576, "seq_len": 4096},
}
CONFIG = CONFIGS["d20"]
L2_NOTE = "inputs larger than L2 (multi-GB activations per micro-step); no flush"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- common
def dist_setup(want_gpus: int):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != want_gpus:
        raise SystemExit(f"--gpus {want_gpus} but WORLD_SIZE={world}; launch with torchrun for N>1")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    return rank, world, local, dev


def max_over_ranks(x: float, dev) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier_sync(dev):
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(dev)


# ----------------------------------------------------------------------------- ours
def run_ours(args) -> dict:
    import contextlib

    import torch
    from trainium_frontier_b200 import ops
    library = args.impl == "library"
    with (ops.oracle_mode() if library else contextlib.nullcontext()):
        out = _run_ours(args)
    if library:
        out["impl"] = "library"
        out["dtype"] = "bf16 (this framework's model and engine with every op on its PyTorch oracle: cuBLAS GEMMs, SDPA, eager elementwise)"
        out["gpu_launches"] = 0
    return out


def _run_ours(args) -> dict:
    import torch
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.ops import _ext
    from trainium_frontier_b200.train import Trainer
    rank, world, local, dev = dist_setup(args.gpus)
    CONFIG = CONFIGS[args.preset]
    per_gpu_tokens = CONFIG["global_batch"] // world
    rows_micro = min(args.micro_rows, per_gpu_tokens // CONFIG["seq_len"])
    cfg = preset(args.preset, device_batch_size=rows_micro, pack_factor=1, progress_mode="steps",
                 num_steps=10 ** 6, grad_sync=args.grad_sync, clip_order="global", seed=1234, tp=args.tp)
    tr = Trainer(cfg, dev, rank, world)
    n_params = sum(p.numel() for p in tr.model.parameters())
    # device-resident inputs for the kernel-only timing
    staged = []
    for _ in range(tr.grad_accum):
        r = tr.loader.next().clone()
        staged.append((r[:, :-1], r[:, 1:]))

    def device_step():
        from trainium_frontier_b200.optim.schedules import apply_schedules
        tr.engine.forward_backward(staged)
        tr.engine.sync_and_clip()
        apply_schedules(cfg, tr.opt, tr.step_idx, tr.progress(0.0))
        tr.engine.optimizer_step()
        tr.step_idx += 1

    for _ in range(args.warmup):
        device_step()
    _ext.check_errors(dev)
    barrier_sync(dev)
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = _ext.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(dev)
    start.record()
    for _ in range(args.steps):
        device_step()
    end.record()
    barrier_sync(dev)
    launches = _ext.launch_count() - launches0
    clk = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms, dev)
    _ext.check_errors(dev)
    # end-to-end through the public API (H2D of each step's rows, D2H of its loss)
    barrier_sync(dev)
    t0 = time.perf_counter()
    losses = []
    for _ in range(args.steps):
        losses.append(tr.train_step())
    barrier_sync(dev)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    e2e_ms = max_over_ranks(e2e_ms, dev)
    tok = CONFIG["global_batch"]
    out = {
        "metric": METRIC, "value": tok / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf(1.1) token stream, BOS=0 docs of geometric mean length 200; random-init weights)",
        "config": dict(CONFIG, parallelism=f"dp{world}" if args.tp == 1 else f"tp{args.tp}xdp{world // args.tp}",
                       micro_batch_rows=rows_micro, grad_accum=tr.grad_accum, l2=L2_NOTE),
        "detail": {"grad_sync": tr.engine.grad_sync, "n_params": n_params, "clip_order": "global"},
        "e2e": {"value": tok / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": tr.h2d_bytes_per_step, "d2h_bytes_per_step": 4,
                "api": "trainium_frontier_b200.train.Trainer.train_step"},
        "gpu_launches": launches,
        "clocks": clk,
        "loss_last": losses[-1],
        "impl": "ours",
    }
    return out


# ----------------------------------------------------------------------------- reference
def zipf_rows(n_rows: int, seq_len: int, seed: int, vocab: int = 8192, s: float = 1.1,
              mean_doc: float = 200.0):
    """[n_rows, seq_len + 1] int32 rows of the benchmark's token statistics, written with
    numpy only so the reference process maps nothing of this framework: ids Zipf(s) over
    [1, vocab) by inverse CDF, a BOS (id 0) opening every document, document lengths
    geometric with mean ``mean_doc``, documents concatenated and cut into rows."""
    import numpy as np
    rng = np.random.default_rng(seed)
    k = np.arange(1, vocab, dtype=np.float64)
    cdf = np.cumsum(k ** -s)
    cdf /= cdf[-1]
    n = n_rows * (seq_len + 1)
    toks = (np.searchsorted(cdf, rng.random(n), side="right") + 1).clip(1, vocab - 1)
    starts = np.cumsum(rng.geometric(1.0 / mean_doc, size=n // 8 + 16) + 1) - 1
    toks[0] = 0
    toks[starts[starts < n]] = 0
    return toks.astype(np.int32).reshape(n_rows, seq_len + 1)


def run_reference(args) -> dict:
    """The unmodified reference module (installed under baseline/_ref) driven through its
    own GPT / init_weights / torch.compile(inductor) / setup_optimizer / clip /
    sync_gradients (per-parameter all-reduce) / MuonAdamW.step path, as its main() does
    (train.py:5846-5885 build, :5999-6258 step loop, :4412-4420 sync).  Nothing of this
    framework is imported here: token rows come from ``zipf_rows`` (numpy)."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "train.py")):
        return {"impl": "reference", "unavailable": "baseline/_ref not installed"}
    import torch
    rank, world, local, dev = dist_setup(args.gpus)
    sys.path.insert(0, ref_dir)
    saved_argv = sys.argv
    sys.argv = ["train.py"]
    import prepare as rprep  # noqa: E402,F401
    import train as rtrain  # noqa: E402
    sys.argv = saved_argv
    CONFIG = CONFIGS[args.preset]
    # the plain family at the preset's shape, through the reference's own globals / API
    rtrain.DEPTH, rtrain.N_EMBD = {"d20": (20, 1280), "d12": (12, 768), "d26": (26, 1664)}[args.preset]
    rtrain.SEQ_LEN = CONFIG["seq_len"]
    rtrain.TOTAL_BATCH_SIZE = CONFIG["global_batch"]
    rtrain.USE_VE = False
    rtrain.USE_NGRAM_VE = False
    rtrain.USE_LOCAL_CONV = False
    rtrain.USE_QK_SHIFT = False
    rtrain.COMPUTE_DTYPE = rtrain.compute_dtype_for(dev)
    rtrain.PACK_FACTOR = 1
    per_gpu_rows = CONFIG["global_batch"] // (CONFIG["seq_len"] * world)
    rows_micro = min(args.ref_micro_rows or args.micro_rows, per_gpu_rows)

    def build(rows):
        rtrain.DEVICE_BATCH_SIZE = rows
        torch.manual_seed(42)
        model = rtrain.GPT(rtrain.build_config())
        model.init_weights()
        model.to(dev)
        return model

    def stage(rows, n, seed):
        blk = torch.from_numpy(zipf_rows(rows * n, CONFIG["seq_len"], seed))
        out = []
        for i in range(n):
            r = blk[i * rows:(i + 1) * rows].to(dev, non_blocking=False)
            out.append((r[:, :-1].contiguous(), r[:, 1:].long().contiguous()))
        return out

    # Largest micro-batch (starting at this framework's) whose warm-up fits in memory.
    while True:
        grad_accum = CONFIG["global_batch"] // (rows_micro * CONFIG["seq_len"] * world)
        orig = build(rows_micro)
        model = torch.compile(orig, backend="inductor", dynamic=False)
        opt = orig.setup_optimizer()
        cached = [m for m in orig.modules() if isinstance(m, rtrain.Linear)]
        clip_main, _clip_ng = rtrain.split_clip_params(orig)
        staged = stage(rows_micro, grad_accum, 1234 + 7919 * (rank + 1))

        def step(batches, i):
            opt.zero_grad(set_to_none=True)
            last = None
            for x, y in batches:
                loss = model(x, y)
                last = loss.detach()
                (loss / grad_accum).backward()
            torch.nn.utils.clip_grad_norm_(clip_main, rtrain.GRAD_CLIP, foreach=True)
            rtrain.sync_gradients(model)
            lrm = rtrain.lr_multiplier(i, elapsed=0.0, max_train_seconds=rtrain.MAX_TRAIN_SECONDS)
            for group in opt.param_groups:
                group["lr"] = group["initial_lr"] * lrm
                if group["kind"] == "muon":
                    group["momentum"] = rtrain.muon_momentum(i, 0.0)
                    group["weight_decay"] = rtrain.WEIGHT_DECAY
            opt.step()
            for m in cached:
                m.refresh_weight_cache(rtrain.COMPUTE_DTYPE)
            return last

        oom = 0
        try:
            step(staged, 0)
        except torch.cuda.OutOfMemoryError:
            oom = 1
        # every rank takes the same branch
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([oom], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            oom = int(t.item())
        if not oom or rows_micro == 1:
            break
        del model, orig, opt, cached, clip_main, staged
        torch._dynamo.reset()
        torch.cuda.empty_cache()
        rows_micro //= 2

    for i in range(1, args.warmup):
        step(staged, i)
    barrier_sync(dev)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(dev)
    start.record()
    for i in range(args.steps):
        step(staged, args.warmup + i)
    end.record()
    barrier_sync(dev)
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, dev)
    # end to end: fresh rows each step, copied host->device from pinned memory, loss read
    # back.  The reference's step is seconds to tens of seconds, so this loop is capped at
    # two steps to bound the arm's time.
    n_e2e = min(args.steps, 2)
    host = [torch.from_numpy(zipf_rows(rows_micro * grad_accum, CONFIG["seq_len"], 99 + 13 * rank + i)).pin_memory()
            for i in range(n_e2e)]
    barrier_sync(dev)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        bs = []
        for j in range(grad_accum):
            r = host[i][j * rows_micro:(j + 1) * rows_micro].to(dev, non_blocking=True)
            bs.append((r[:, :-1].contiguous(), r[:, 1:].long().contiguous()))
        float(step(bs, args.warmup + args.steps + i).item())
    barrier_sync(dev)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0 / n_e2e, dev)
    tok = CONFIG["global_batch"]
    return {
        "metric": METRIC, "value": tok / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 weights; block GEMMs in fp32 (the reference's shape-[1] fp32 resid/x0 lambdas promote its residual stream to fp32 on CUDA, TF32 off)",
        "data": "synthetic (seeded Zipf(1.1) token stream, BOS=0 docs of geometric mean length 200; random-init weights)",
        "config": dict(CONFIG, parallelism=f"dp{world}", micro_batch_rows=rows_micro, grad_accum=grad_accum,
                       l2=L2_NOTE),
        "detail": {"path": "reference train.py: torch.compile(inductor) + SDPA + eager Muon + per-parameter all_reduce",
                   "grad_sync": "per-parameter all_reduce", "requested_micro_rows": args.ref_micro_rows or args.micro_rows},
        "e2e": {"value": tok / (e2e_ms / 1000.0), "unit": "tokens/s", "ms_per_step": e2e_ms, "steps": n_e2e,
                "h2d_bytes_per_step": grad_accum * rows_micro * (CONFIG["seq_len"] + 1) * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": 0,
        "clocks": clk,
        "impl": "reference",
    }


def run_infer(args) -> dict:
    from trainium_frontier_b200.utils import infer_bench
    if args.impl == "reference" and not os.path.exists(os.path.join(ROOT, "baseline", "_ref", "train.py")):
        return {"impl": "reference", "unavailable": "baseline/_ref not installed"}
    rank, world, local, dev = dist_setup(args.gpus)
    clocks = ClockSampler(local)
    clocks.start()
    out = infer_bench.run(args, args.impl, ROOT, rank, world, local, dev)
    out["clocks"] = clocks.stop()
    if args.impl == "ours":
        from trainium_frontier_b200.ops import _ext
        out["gpu_launches"] = _ext.launch_count()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "library"],
                    help="ours: the sm_100a kernels; reference: the reference's own CUDA path; library: this "
                         "framework's model with every op on its PyTorch oracle (a bf16 library comparator)")
    ap.add_argument("--micro-rows", type=int, default=0,
                    help="sequences per micro-step per GPU (default: 32 at seq 2048, 4 for d26 at seq 4096)")
    ap.add_argument("--ref-micro-rows", type=int, default=0,
                    help="reference arm sequences per micro-step (default: the same as --micro-rows; halved "
                         "until its first step fits in memory)")
    ap.add_argument("--grad-sync", default="auto")
    ap.add_argument("--preset", default="d20", choices=sorted(CONFIGS), help="model / batch configuration")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel degree (ours; DP = N / tp)")
    ap.add_argument("--workload", default="train", choices=["train", "infer"],
                    help="train: the d20 pretraining step (default); infer: held-out eval + KV-cache decode")
    args = ap.parse_args()
    if args.micro_rows <= 0:
        args.micro_rows = 4 if args.preset == "d26" else 32
    if args.warmup < 3:
        args.warmup = 3
    try:
        if args.workload == "infer":
            out = run_infer(args)
        else:
            out = run_reference(args) if args.impl == "reference" else run_ours(args)
    except Exception as e:  # noqa: BLE001
        if args.impl == "reference":
            out = {"impl": "reference", "unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
        else:
            raise
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps(out), flush=True)
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
    except Exception:
        pass


if __name__ == "__main__":
    main()
