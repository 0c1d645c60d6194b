"""Autoresearch loop: a fixed 5-minute single-GPU training run of a small plain GPT that
prints ``val_bpb`` -- the quick A/B harness of the reference's ``autoresearch/train.py``
(depth 6, width 640 = aspect 96 rounded to the 128 head dim, seq 2048, 131,072-token
batches of 16 rows, softcap 11, rotary base 2e6, its own learning rates, no weight decay,
no warmdown).

    python -m trainium_frontier_b200.research.autoresearch [--time-budget 300] [--flag value ...]

Any trainer flag can be appended to try a variant (``--matrix-lr 0.05``); the run ends
after ``--time-budget`` seconds of training (startup excluded as in the trainer), then
evaluates held-out bpb and prints the summary block plus one ``val_bpb: ...`` line.
Differences from the reference loop: the Muon momentum ramp is the trainer's (0.85 ->
0.95 over 300 steps), and the data is the seeded synthetic stream.
"""
from __future__ import annotations

import argparse
import dataclasses

from ..config import build_parser, preset, validate
from ..train import run


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(add_help=False)
    ap.add_argument("--time-budget", type=int, default=300)
    known, rest = ap.parse_known_args(argv)
    base = preset("autoresearch", max_train_seconds=known.time_budget, num_steps=10 ** 9)
    ns = build_parser(base).parse_args(rest)
    cfg = dataclasses.replace(base, **{f.name: getattr(ns, f.name) for f in dataclasses.fields(base)})
    validate(cfg)
    summary = run(cfg)
    if "val_bpb" in summary:
        print(f"val_bpb: {summary['val_bpb']:.6f}")


if __name__ == "__main__":
    main()
