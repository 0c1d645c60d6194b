"""Operator census of one training step: every ATen op dispatched and every sm_100a kernel
call, by name and phase (forward+backward, gradient sync+clip, optimizer).

ATen ops are observed with ``TorchDispatchMode`` (the real op stream, not a count read
off the source) and classed as matmul, view (metadata only, launches nothing) or
elementwise/reduce (the launches a fused kernel removes).  Native kernel calls come from
the extension's per-entry-point counter.  On a GPU a phase's ``launch_bound`` figure is
the number of launches it issues outside the tensor-core GEMMs; on the CPU the step runs
the fp32 oracle, so only ATen ops appear.

The reference takes the same census of its Muon step alone
(``research/scratch/muon_dispatch_census.py``) to size its optimizer fusion; this one
covers the whole step.

    python -m trainium_frontier_b200.utils.op_census --preset tiny --depth 2 --device cpu
    python -m trainium_frontier_b200.utils.op_census --preset d20 --rows 2 --device cuda
"""
from __future__ import annotations

import argparse
import json
from collections import Counter

import torch
from torch.utils._python_dispatch import TorchDispatchMode

MATMUL_OPS = {"mm", "bmm", "addmm", "baddbmm", "matmul", "linear", "_scaled_mm",
              "convolution", "convolution_backward",
              "_scaled_dot_product_flash_attention", "_scaled_dot_product_efficient_attention",
              "_scaled_dot_product_cudnn_attention", "_flash_attention_forward",
              "_flash_attention_backward", "_scaled_dot_product_flash_attention_backward"}
VIEW_OPS = {"view", "reshape", "_unsafe_view", "transpose", "permute", "t", "expand",
            "unbind", "select", "slice", "detach", "alias", "squeeze", "unsqueeze",
            "as_strided", "is_same_size", "split", "split_with_sizes", "chunk", "narrow",
            "unflatten", "flatten", "view_as", "lift_fresh", "_reshape_alias", "diagonal",
            "real", "empty", "empty_like", "empty_strided", "new_empty", "new_empty_strided",
            "_local_scalar_dense", "set_", "record_stream"}


def op_class(name: str) -> str:
    """'matmul', 'view' or 'elementwise' for an ATen overload packet name such as 'mm'."""
    base = name.split(".")[0]
    if base in MATMUL_OPS:
        return "matmul"
    if base in VIEW_OPS:
        return "view"
    return "elementwise"


class Census(TorchDispatchMode):
    """Counts every ATen op that reaches the dispatcher while active."""

    def __init__(self):
        super().__init__()
        self.ops: Counter = Counter()

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops[func.overloadpacket.__name__] += 1
        return func(*args, **(kwargs or {}))


def _native_counts() -> dict[str, int]:
    from ..ops import _ext
    return _ext.launch_counts_by_name()


def census_phase(fn) -> dict:
    """Run ``fn()`` under the census; returns per-class ATen counts, the ATen op table and
    the native kernel calls it made."""
    before = _native_counts()
    with Census() as c:
        fn()
    after = _native_counts()
    native = {k: v - before.get(k, 0) for k, v in after.items() if v - before.get(k, 0)}
    classes = Counter()
    for name, n in c.ops.items():
        classes[op_class(name)] += n
    return {
        "aten_matmul": classes["matmul"],
        "aten_elementwise": classes["elementwise"],
        "aten_view": classes["view"],
        "native": sum(native.values()),
        "launch_bound": classes["elementwise"] + sum(v for k, v in native.items()
                                                     if not k.startswith("gemm")),
        "aten_ops": dict(c.ops.most_common()),
        "native_ops": dict(sorted(native.items(), key=lambda kv: -kv[1])),
    }


def step_census(trainer, batches, schedules=None) -> dict:
    """Census of one optimizer step of ``trainer`` on ``batches`` [(x, y), ...], by phase."""
    eng = trainer.engine
    out = {"fwd_bwd": census_phase(lambda: eng.forward_backward(batches)),
           "sync_clip": census_phase(lambda: eng.sync_and_clip())}
    if schedules is not None:
        schedules()
    out["optimizer"] = census_phase(lambda: eng.optimizer_step())
    trainer.step_idx += 1
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--depth", type=int, default=0, help="override the preset's depth")
    ap.add_argument("--rows", type=int, default=2)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--top", type=int, default=12)
    ap.add_argument("--json", default="")
    args = ap.parse_args(argv)
    from ..config import preset
    from ..optim.schedules import apply_schedules
    from ..train import Trainer
    dev = torch.device(args.device, 0) if args.device == "cuda" else torch.device(args.device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    kw = {"depth": args.depth} if args.depth else {}
    cfg0 = preset(args.preset, **kw)
    cfg = preset(args.preset, device_batch_size=args.rows, pack_factor=1, progress_mode="steps",
                 num_steps=10 ** 6, total_batch_size=args.rows * cfg0.seq_len, **kw)
    tr = Trainer(cfg, dev)
    r = tr.loader.next().clone()
    batches = [(r[:, :-1], r[:, 1:])]
    for _ in range(args.warmup):
        tr.engine.forward_backward(batches)
        tr.engine.sync_and_clip()
        tr.engine.optimizer_step()
        tr.step_idx += 1
    res = step_census(tr, batches, lambda: apply_schedules(cfg, tr.opt, tr.step_idx, 0.0))
    if dev.type == "cuda":
        torch.cuda.synchronize()
    for phase, d in res.items():
        print(f"{phase:10s} matmul {d['aten_matmul']:5d}  elementwise {d['aten_elementwise']:5d}  "
              f"view {d['aten_view']:5d}  native {d['native']:5d}  launch-bound {d['launch_bound']:5d}")
        top = list(d["aten_ops"].items())[:args.top]
        print("           aten:", ", ".join(f"{k}×{v}" for k, v in top))
        if d["native_ops"]:
            print("           native:", ", ".join(f"{k}×{v}" for k, v in d["native_ops"].items()))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(res, f, indent=1)
    return res


if __name__ == "__main__":
    main()
