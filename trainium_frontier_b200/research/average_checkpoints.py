"""Average N checkpoints (out/final.pt layout) into one static checkpoint.

    python -m trainium_frontier_b200.research.average_checkpoints --out avg.pt a.pt b.pt [--ema|--raw]
    python -m trainium_frontier_b200.research.average_checkpoints --selftest

Same contract as the reference's ``research/average_checkpoints.py``: every input must
have the same ``model_config`` and state keys/shapes; ``ema_state`` is averaged when every
input carries one (``auto``), raw ``model_state`` otherwise, and a mix is refused when
``--ema`` is forced.  The result is a normal payload (``model_state``, ``model_config``,
``toggles``, ``meta``) that ``load_for_eval`` reads unchanged.  CPU only; the average is
accumulated in fp64 and cast back to each tensor's dtype.
"""
from __future__ import annotations

import argparse
import sys
import tempfile
from pathlib import Path

import torch


def _load(p) -> dict:
    return torch.load(str(p), map_location="cpu", weights_only=True)


def average_checkpoints(paths: list, use_ema: str = "auto") -> dict:
    if not paths:
        raise ValueError("no input checkpoints")
    if use_ema not in ("auto", "ema", "raw"):
        raise ValueError(f"use_ema must be auto / ema / raw, got {use_ema!r}")
    pl = [_load(p) for p in paths]
    cfg0 = pl[0]["model_config"]
    for p, x in zip(paths[1:], pl[1:]):
        if x["model_config"] != cfg0:
            raise ValueError(f"model_config differs: {paths[0]} vs {p}")
    have = [("ema_state" in x) for x in pl]
    if use_ema == "ema" and not all(have):
        raise ValueError(f"--ema requested but missing in: {[str(p) for p, h in zip(paths, have) if not h]}")
    key = "ema_state" if (use_ema == "ema" or (use_ema == "auto" and all(have))) else "model_state"
    if use_ema == "auto" and any(have) and not all(have):
        print("WARNING: not every input has ema_state; averaging model_state", file=sys.stderr)
    keys = list(pl[0][key].keys())
    for p, x in zip(paths[1:], pl[1:]):
        if set(x[key].keys()) != set(keys):
            raise ValueError(f"state keys differ: {paths[0]} vs {p}")
        for k in keys:
            if x[key][k].shape != pl[0][key][k].shape:
                raise ValueError(f"shape of {k} differs: {paths[0]} vs {p}")
    avg = {}
    n = float(len(pl))
    for k in keys:
        acc = torch.zeros(pl[0][key][k].shape, dtype=torch.float64)
        for x in pl:
            acc += x[key][k].double()
        avg[k] = (acc / n).to(pl[0][key][k].dtype)
    meta = dict(pl[0].get("meta", {}))
    meta.update({"averaged_from": [str(p) for p in paths], "averaged_key": key})
    return {"model_state": avg, "model_config": cfg0, "toggles": pl[0].get("toggles", {}), "meta": meta}


def _selftest() -> None:
    cfg = {"sequence_len": 8, "vocab_size": 16, "n_layer": 1, "n_head": 1, "n_embd": 4, "mlp_ratio": 4,
           "attn_scale": 0.0, "n_kv_heads": 0}
    with tempfile.TemporaryDirectory() as d:
        ps = []
        for i in range(3):
            p = Path(d) / f"c{i}.pt"
            torch.save({"model_state": {"w": torch.full((2, 2), float(i))}, "model_config": cfg, "toggles": {},
                        "meta": {"step": i}, "ema_state": {"w": torch.full((2, 2), 10.0 + i)}}, p)
            ps.append(p)
        out = average_checkpoints(ps)
        assert torch.allclose(out["model_state"]["w"], torch.full((2, 2), 11.0)), "ema average"
        out = average_checkpoints(ps, "raw")
        assert torch.allclose(out["model_state"]["w"], torch.full((2, 2), 1.0)), "raw average"
    print("selftest passed")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("inputs", nargs="*")
    ap.add_argument("--out", default="")
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--ema", action="store_const", const="ema", dest="mode")
    g.add_argument("--raw", action="store_const", const="raw", dest="mode")
    ap.add_argument("--selftest", action="store_true")
    a = ap.parse_args(argv)
    if a.selftest:
        return _selftest()
    if not a.inputs or not a.out:
        ap.error("inputs and --out are required")
    payload = average_checkpoints([Path(p) for p in a.inputs], a.mode or "auto")
    Path(a.out).parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, a.out)
    print(f"wrote {a.out} ({payload['meta']['averaged_key']} of {len(a.inputs)} checkpoints)")


if __name__ == "__main__":
    main()
