"""Score ONE checkpoint under every evaluation definition in use, in one table.

    python -m trainium_frontier_b200.research.reconcile_eval --checkpoint out/final.pt [--device cuda]
    python -m trainium_frontier_b200.research.reconcile_eval --dry-run

The cells are {raw weights, EMA weights} x {seq 2048, seq 1024} (plus ``--cell
name:weights:seq``), the matrix the reference's ``research/reconcile_eval.py`` evaluates,
each through the trusted ``evaluate_bpb`` so every reported bpb can be labelled with the
definition that produced it.  EMA cells are skipped when the checkpoint has no
``ema_state``.  Prints one JSON object per cell.
"""
from __future__ import annotations

import argparse
import json
import time

import torch

BASE_CELLS = [("raw-2048", "raw", 2048), ("ema-2048", "ema", 2048), ("raw-1024", "raw", 1024),
              ("ema-1024", "ema", 1024)]


def plan_cells(custom: list[str]) -> list[dict]:
    cells = [{"name": n, "weights": w, "seq_len": s} for n, w, s in BASE_CELLS]
    for c in custom:
        n, w, s = c.split(":")
        if w not in ("raw", "ema"):
            raise ValueError(f"cell weights must be raw or ema: {c}")
        cells.append({"name": n, "weights": w, "seq_len": int(s)})
    return cells


def run(checkpoint: str, cells: list[dict], batch_size: int, device, max_tokens: int | None) -> list[dict]:
    from ..checkpoint import load_for_eval, torch_load_weights
    from ..data.synthetic import SyntheticTokenizer
    from ..eval import evaluate_bpb
    payload = torch_load_weights(checkpoint, map_location="cpu")
    has_ema = "ema_state" in payload
    rows = []
    models = {}
    for cell in cells:
        if cell["weights"] == "ema" and not has_ema:
            rows.append(dict(cell, skipped="checkpoint has no ema_state"))
            continue
        if cell["weights"] not in models:
            models[cell["weights"]] = load_for_eval(checkpoint, device, prefer_ema=cell["weights"] == "ema")
        t0 = time.monotonic()
        res = evaluate_bpb(models[cell["weights"]], SyntheticTokenizer(), batch_size, cell["seq_len"], device,
                           max_tokens=max_tokens)
        rows.append(dict(cell, val_bpb=res["val_bpb"], num_tokens=res["num_tokens"], num_bytes=res["num_bytes"],
                         seconds=time.monotonic() - t0))
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--checkpoint", default="")
    ap.add_argument("--device", default="")
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--max-tokens", type=int, default=1 << 20)
    ap.add_argument("--cell", action="append", default=[], help="extra cell name:raw|ema:seq_len")
    ap.add_argument("--dry-run", action="store_true", help="print the cell plan only")
    a = ap.parse_args(argv)
    cells = plan_cells(a.cell)
    if a.dry_run or not a.checkpoint:
        for c in cells:
            print(json.dumps(c))
        return
    dev = torch.device(a.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    for row in run(a.checkpoint, cells, a.batch_size, dev, a.max_tokens):
        print(json.dumps(row))


if __name__ == "__main__":
    main()
