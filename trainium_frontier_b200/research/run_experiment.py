"""Experiment runner: launch the trainer, parse its final ``key: value`` summary, append
one JSON row to an experiment log.

    python -m trainium_frontier_b200.research.run_experiment --label my-run --description "..." \
        [--nproc-per-node 8] [--log experiment-log.jsonl] -- [trainer flags ...]

The trainer (``python -m trainium_frontier_b200.train``) prints a ``---`` line followed by
``key: value`` lines at the end of a run (val_bpb, causality, steps, tokens, params); those
become the row's ``summary``, next to the label, description, launch command, wall time,
exit status (``ok`` / ``crash``) and the last 40 log lines of a crashed run.  Mirrors the
reference's ``research/run_experiment.py`` (one process per accelerator, torchrun for
N > 1, rendezvous on 127.0.0.1).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from datetime import datetime, timezone


def parse_summary(text: str) -> dict:
    out = {}
    lines = text.splitlines()
    try:
        start = len(lines) - 1 - lines[::-1].index("---")
    except ValueError:
        start = -1
    for ln in lines[start + 1:]:
        if ": " not in ln:
            continue
        k, v = ln.split(": ", 1)
        k = k.strip()
        if not k or " " in k:
            continue
        v = v.strip()
        for cast in (int, float):
            try:
                v = cast(v)
                break
            except ValueError:
                pass
        else:
            if v in ("True", "False"):
                v = v == "True"
        out[k] = v
    return out


def build_command(nproc: int, trainer_args: list[str], port: int) -> list[str]:
    if nproc <= 1:
        return [sys.executable, "-m", "trainium_frontier_b200.train"] + trainer_args
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
            "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "trainium_frontier_b200.train"] + trainer_args


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--label", required=True)
    ap.add_argument("--description", default="")
    ap.add_argument("--nproc-per-node", type=int, default=1)
    ap.add_argument("--port", type=int, default=29555)
    ap.add_argument("--log", default="experiment-log.jsonl")
    ap.add_argument("--timeout", type=int, default=4 * 3600)
    ap.add_argument("trainer_args", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    targs = a.trainer_args[1:] if a.trainer_args[:1] == ["--"] else a.trainer_args
    cmd = build_command(a.nproc_per_node, targs, a.port)
    t0 = time.monotonic()
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=a.timeout, env=dict(os.environ))
        rc, text = p.returncode, p.stdout + p.stderr
    except subprocess.TimeoutExpired as e:
        rc, text = -9, (e.stdout or "") if isinstance(e.stdout, str) else ""
    row = {"label": a.label, "description": a.description, "command": cmd,
           "started_utc": datetime.now(timezone.utc).isoformat(timespec="seconds"),
           "wall_seconds": round(time.monotonic() - t0, 1), "status": "ok" if rc == 0 else "crash",
           "returncode": rc, "summary": parse_summary(text)}
    if rc != 0:
        row["log_tail"] = text.splitlines()[-40:]
    with open(a.log, "a", encoding="utf-8") as f:
        f.write(json.dumps(row) + "\n")
    print(json.dumps(row["summary"] if rc == 0 else row, indent=1))
    if rc != 0:
        raise SystemExit(rc)


if __name__ == "__main__":
    main()
