"""Held-out bpb parity at equal training tokens on one GPU: this framework against the
reference's own CUDA path, same model, same initial weights, same batches.

    python -m trainium_frontier_b200.utils.parity_bench [--preset d12] [--steps 200]
        [--rows 16] [--eval-tokens 1048576] [--json out.json]

* The reference is the unmodified ``baseline/_ref/train.py`` imported as a module (its
  ``GPT``, ``init_weights``, ``setup_optimizer``, ``clip_grad_norm_`` over its clip set
  and ``MuonAdamW.step``, eager), configured through its globals to the plain member of
  the preset's shape; its initial ``state_dict`` is loaded into this framework's model
  (the key layouts are shared), so both arms start from the same weights.
* Both arms see the same seeded synthetic Zipf batches and the same per-step learning
  rate / momentum / weight decay (constant lr, the reference's momentum warm-up, weight
  decay decaying linearly to zero over the run), in bf16 compute on the GPU.
* After training both are scored by the same ``evaluate_bpb`` over ``--eval-tokens``
  held-out tokens.  The JSON line reports both bpb values, their difference and the
  reference's published seed-to-seed spread of 0.0061 bpb (max - min over seeds).

Reference counterparts: its training step (``train.py:5999-6258``) and trusted scoring
(``prepare.py:595-659``, run after training at ``train.py:6277-6306``).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
SEED_SPREAD_BPB = 0.0061  # the reference's max - min held-out bpb over seeds (trn2 results)
SHAPES = {"d12": (12, 768, 2048), "d20": (20, 1280, 2048), "tiny": (4, 256, 256)}


def import_reference():
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "train.py")):
        raise SystemExit("reference not installed under baseline/_ref")
    sys.path.insert(0, ref_dir)
    argv = sys.argv
    sys.argv = ["train.py"]
    try:
        import train as rtrain  # noqa: E402
    finally:
        sys.argv = argv
    return rtrain


def batches(n: int, rows: int, T: int, seed: int, dev):
    from trainium_frontier_b200.data.loader import PackedRowLoader
    ld = PackedRowLoader(rows, T, torch.device("cpu"), "train", seed=seed, rank=0)
    out = []
    for _ in range(n):
        r = ld.next().clone().to(dev)
        out.append((r[:, :-1].contiguous(), r[:, 1:].long().contiguous()))
    return out


def schedule(groups, step: int, n_steps: int, momentum_fn, wd: float) -> None:
    prog = step / n_steps
    for g in groups:
        g["lr"] = g["initial_lr"]
        if g["kind"] == "muon":
            g["momentum"] = momentum_fn(step, prog)
            g["weight_decay"] = wd * (1.0 - prog)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="d12", choices=sorted(SHAPES))
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--rows", type=int, default=16, help="sequences per step (one micro-step)")
    ap.add_argument("--eval-tokens", type=int, default=1 << 20)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", default="")
    ap.add_argument("--device", default="cuda", help="cuda (bf16) or cpu (fp32, a quick functional check)")
    args = ap.parse_args()
    dev = torch.device(args.device, 0) if args.device == "cuda" else torch.device("cpu")
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    depth, width, T = SHAPES[args.preset]

    # ---- reference arm: its own model, init and optimizer
    rtrain = import_reference()
    rtrain.DEPTH, rtrain.N_EMBD, rtrain.SEQ_LEN = depth, width, T
    rtrain.HEAD_DIM = 64 if args.preset == "tiny" else 128
    rtrain.USE_VE = False
    rtrain.USE_NGRAM_VE = False
    rtrain.USE_LOCAL_CONV = False
    rtrain.USE_QK_SHIFT = False
    rtrain.COMPUTE_DTYPE = rtrain.compute_dtype_for(dev)
    torch.manual_seed(args.seed)
    ref = rtrain.GPT(rtrain.build_config())
    ref.init_weights()
    if args.preset == "tiny":  # the tiny member's rotary base
        cos, sin = ref._precompute_rotary_embeddings(T, rtrain.HEAD_DIM, base=10000)
        ref.cos.copy_(cos)
        ref.sin.copy_(sin)
    init_state = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    ref.to(dev)
    opt_r = ref.setup_optimizer()
    cached = [m for m in ref.modules() if isinstance(m, rtrain.Linear)]
    clip_main, _ = rtrain.split_clip_params(ref)

    # ---- this framework: same shape, the reference's initial weights
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.eval import evaluate_bpb
    from trainium_frontier_b200.optim.schedules import muon_momentum
    from trainium_frontier_b200.train import Trainer
    cfg = preset(args.preset if args.preset != "tiny" else "tiny", device_batch_size=args.rows, pack_factor=1,
                 total_batch_size=args.rows * T, progress_mode="steps", num_steps=args.steps, seed=args.seed,
                 clip_order="local")
    tr = Trainer(cfg, dev, build_loader=False)
    with torch.no_grad():
        missing = tr.model.load_state_dict({k: v.to(dev) for k, v in init_state.items()}, strict=False)
    assert not missing.missing_keys, missing.missing_keys
    tr.engine.layout.refresh_bf16()

    data = batches(args.steps, args.rows, T, 4321 + args.seed, dev)
    hist_r, hist_o = [], []
    t0 = time.perf_counter()
    for i, (x, y) in enumerate(data):
        # reference step (its stock eager path)
        opt_r.zero_grad(set_to_none=True)
        loss = ref(x, y)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(clip_main, rtrain.GRAD_CLIP, foreach=True)
        schedule(opt_r.param_groups, i, args.steps, rtrain.muon_momentum, rtrain.WEIGHT_DECAY)
        opt_r.step()
        for m in cached:
            m.refresh_weight_cache(rtrain.COMPUTE_DTYPE)
        hist_r.append(float(loss))
    t_ref = time.perf_counter() - t0
    t0 = time.perf_counter()
    for i, (x, y) in enumerate(data):
        lo = tr.engine.forward_backward([(x, y)])
        tr.engine.sync_and_clip()
        schedule(tr.opt.param_groups, i, args.steps, lambda s, p: muon_momentum(cfg, s, p), cfg.weight_decay)
        tr.engine.optimizer_step()
        hist_o.append(float(lo))
    t_ours = time.perf_counter() - t0
    with torch.no_grad():
        r_ref = evaluate_bpb(ref, None, 8, T, dev, max_tokens=args.eval_tokens)
        r_our = evaluate_bpb(tr.model, None, 8, T, dev, max_tokens=args.eval_tokens)
    out = {
        "metric": "held-out bpb at equal training tokens (same init, same batches)",
        "preset": args.preset, "steps": args.steps, "tokens_per_step": args.rows * T,
        "train_tokens": args.steps * args.rows * T, "eval_tokens": r_our["num_tokens"],
        "bpb_reference": r_ref["val_bpb"], "bpb_ours": r_our["val_bpb"],
        "bpb_diff": r_our["val_bpb"] - r_ref["val_bpb"], "seed_spread_bpb": SEED_SPREAD_BPB,
        "loss_first": [hist_r[0], hist_o[0]], "loss_last": [hist_r[-1], hist_o[-1]],
        "train_s": {"reference": t_ref, "ours": t_ours},
        "dtype": "bf16 compute (reference: its CUDA path, fp32 block GEMMs)",
        "data": "synthetic (seeded Zipf(1.1) token stream; shared random init)",
    }
    print(json.dumps(out))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
