"""Training entry point: ``python -m trainium_frontier_b200.train [--flags]`` or
``torchrun --nproc-per-node N -m trainium_frontier_b200.train``.

Mirrors the reference's ``main()`` (``train.py:4930-6457``): flags with
``NEURON_COMPETITION_R1_*`` env overrides, gradient accumulation to a fixed global
batch, wall-clock (or step) schedules, per-step health/deadline agreement across
ranks, rank-0 ``out/final.pt`` plus barrier, then causality check + held-out bpb and a
``key: value`` summary.  ``Trainer`` is the public API the benchmark drives: one
``train_step()`` = one optimizer step including the host->device copies of the step's
token rows and the device->host read of its loss.
"""
from __future__ import annotations

import gc
import json
import math
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

from . import checkpoint as ckpt
from .config import (TRAIN_STARTUP_STEPS_EXCLUDED, RunConfig, parse_args, parse_float_tuple)
from .data import synthetic as syn
from .data.loader import PackedRowLoader
from .engine import TrainEngine
from .eval import causality_check, evaluate_bpb
from .models.gpt import GPT
from .optim.muon_adamw import setup_optimizer
from .optim.schedules import apply_schedules, batch_ramp_grad_accum
from .parallel.ddp import grads_finite_, next_loss_scale, unscale_grads_
from .runtime import cleanup_runtime, compute_dtype_for, detect_device_type, init_runtime, print0, synchronize

_PROCESS_STARTED = time.monotonic()


def record_step_boundary(step: int) -> None:
    """Rank-0 append of the step index to NEURON_COMPETITION_R1_STEP_LOG (prepare.py:96-112)."""
    path = os.environ.get("NEURON_COMPETITION_R1_STEP_LOG", "")
    if not path or int(os.environ.get("RANK", "0")) != 0:
        return
    with open(path, "a", encoding="utf-8") as fh:
        fh.write(f"{int(step)}\n")
        fh.flush()
        os.fsync(fh.fileno())


class Trainer:
    """Builds model / optimizer / engine / loader for a RunConfig and runs steps."""

    def __init__(self, cfg: RunConfig, device: torch.device | None = None, rank: int = 0, world_size: int = 1,
                 build_loader: bool = True):
        self.cfg = cfg
        self.device = device or torch.device("cuda" if torch.cuda.is_available() else "cpu")
        self.rank, self.world = rank, world_size
        self.dtype = compute_dtype_for(self.device)
        self.gconf = cfg.model_config()
        torch.manual_seed(cfg.seed)
        model = GPT(self.gconf, cfg)
        model.set_compute_dtype(self.dtype)
        model.init_weights()
        if cfg.init_from:
            ckpt.warm_start_from(cfg.init_from, model)
        self.model = model
        self.tpc = None
        if cfg.tp > 1:
            from .parallel.tensor_parallel import TPContext
            rows = cfg.device_batch_size * cfg.pack_factor * cfg.seq_len
            self.tpc = TPContext(cfg.tp, self.device, rows, self.gconf.n_embd, 2 * self.gconf.n_layer)
            model.enable_tp(self.tpc)
        self.ppc = None
        if cfg.pp > 1:
            from .parallel.pipeline import PipelineContext
            self.ppc = PipelineContext(cfg.pp, self.gconf.n_layer)
            model.enable_pp(self.ppc)
        self.opt = setup_optimizer(model, cfg, compute_dtype=self.dtype)
        self.rows_per_micro = cfg.device_batch_size * cfg.pack_factor
        data_ranks = world_size // cfg.pp          # pipeline stages share their micro-batches
        tokens_per_micro = self.rows_per_micro * cfg.seq_len * data_ranks
        if cfg.total_batch_size % tokens_per_micro:
            raise ValueError(f"total_batch_size={cfg.total_batch_size} must be a multiple of "
                             f"micro tokens x world = {tokens_per_micro}")
        self.grad_accum = cfg.total_batch_size // tokens_per_micro
        self.tokens_per_step = cfg.total_batch_size
        self.engine = TrainEngine(model, self.opt, cfg, self.device, self.grad_accum, cfg.grad_sync)
        self.text_tok = None
        self.loader = PackedRowLoader(self.rows_per_micro, cfg.seq_len, self.device, "train",
                                      rank=rank // cfg.pp, epoch_tokens=cfg.synthetic_epoch_tokens,
                                      epoch_shuffle=cfg.epoch_shuffle,
                                      epoch_shuffle_seed=cfg.epoch_shuffle_seed,
                                      packer=self._text_packer(rank // cfg.pp, data_ranks)) if build_loader else None
        self.step_idx = 0
        self._adamw_applied_last = True   # AdamW gradients are zeroed only after they were applied
        self.loss_scale = cfg.loss_scale
        self.loss_scale_clean = 0
        self.row_weight = None
        if cfg.byte_loss_weight:
            tb = syn.get_token_bytes("cpu", cfg.vocab_size).float().clamp(min=1.0)
            self.byte_w = (tb / tb.mean()).to(self.device)
        else:
            self.byte_w = None

    # ------------------------------------------------------------------ resume
    def resume_state(self) -> dict:
        """Everything an exact continuation needs: weights, optimizer state (including the
        distributed-Muon owner shards of this rank), counters, RNG and the loader cursor."""
        params = list(self.model.parameters())
        index = {id(p): i for i, p in enumerate(params)}

        def cpu(v):
            return v.detach().cpu().clone() if torch.is_tensor(v) else v

        opt_state = {index[id(p)]: {k: cpu(v) for k, v in st.items()} for p, st in self.opt.state.items()
                     if id(p) in index}
        dm = self.engine.dist_muon
        dm_state = {index[k]: {kk: cpu(vv) for kk, vv in st.items()} for k, st in dm.state.items()} \
            if dm is not None else {}
        return {"model_state": {k: v.detach().cpu().clone() for k, v in self.model.state_dict().items()},
                "optimizer": opt_state, "dist_muon": dm_state, "step": self.step_idx,
                "loss_scale": self.loss_scale, "loss_scale_clean": self.loss_scale_clean,
                "loader_batches": self.loader.i if self.loader is not None else 0,
                "rng_cpu": torch.get_rng_state(),
                "rng_cuda": torch.cuda.get_rng_state(self.device) if self.device.type == "cuda" else None,
                "world": self.world, "rank": self.rank}

    def save_resume(self, path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(path.suffix + ".tmp")
        torch.save(self.resume_state(), tmp)
        os.replace(tmp, path)

    def load_resume(self, path) -> None:
        st = torch.load(path, map_location="cpu", weights_only=False)
        if st["world"] != self.world:
            raise ValueError(f"resume file was written by a world of {st['world']} ranks, not {self.world}")
        with torch.no_grad():
            self.model.load_state_dict(st["model_state"], strict=True)   # copies into the flat buffers
        params = list(self.model.parameters())
        for i, d in st["optimizer"].items():
            tgt = self.opt.state[params[i]]
            for k, v in d.items():
                tgt[k] = v.to(self.device) if torch.is_tensor(v) else v
        dm = self.engine.dist_muon
        if dm is not None:
            for i, d in st["dist_muon"].items():
                dm.state[id(params[i])] = {k: v.to(self.device) for k, v in d.items()}
        self.engine.layout.refresh_bf16()
        if self.tpc is not None:
            self.tpc.weights_version += 1
        self.step_idx = st["step"]
        self.loss_scale, self.loss_scale_clean = st["loss_scale"], st["loss_scale_clean"]
        if self.loader is not None:
            for _ in range(st["loader_batches"] - self.loader.i):   # the stream is deterministic
                self.loader.next()
        torch.set_rng_state(st["rng_cpu"])
        if st.get("rng_cuda") is not None and self.device.type == "cuda":
            torch.cuda.set_rng_state(st["rng_cuda"], self.device)

    @property
    def h2d_bytes_per_step(self) -> int:
        return self.grad_accum * self.rows_per_micro * (self.cfg.seq_len + 1) * 4

    def _text_packer(self, rank: int, world: int):
        """Packed rows from ``--text-data`` parquet files tokenized with ``--tokenizer-zip``
        (None: the synthetic stream)."""
        cfg = self.cfg
        if not cfg.text_data:
            return None
        import glob
        from .data.text_loader import TextPacker
        from .data.tokenizer import Tokenizer
        from .harness import CACHE_DIR
        if not cfg.tokenizer_zip:
            raise ValueError("--text-data needs --tokenizer-zip (the tokenizer the text is encoded with)")
        # the model's vocabulary must be the tokenizer's (from_zip checks it)
        cache = os.environ.get("NEURON_COMPETITION_R1_CACHE_DIR", str(CACHE_DIR))
        tok = Tokenizer.from_zip(cfg.tokenizer_zip, os.path.join(cache, "tokenizer"), expected_vocab=cfg.vocab_size)
        self.text_tok = tok
        return TextPacker(tok, sorted(glob.glob(cfg.text_data)), rank, world)

    def eval_tokenizer(self):
        """The tokenizer the post-training evaluation scores with: with ``--text-val-data``,
        the text tokenizer over those held-out parquet files (UTF-8 byte lengths), else
        the synthetic corpus's held-out stream."""
        cfg = self.cfg
        tok = getattr(self, "text_tok", None)
        if tok is None or not cfg.text_val_data:
            return syn.SyntheticTokenizer(cfg.vocab_size)
        import glob
        from .data.text_loader import parquet_documents
        paths = sorted(glob.glob(cfg.text_val_data))
        if not paths:
            raise ValueError(f"--text-val-data {cfg.text_val_data!r} matches no files")
        tok.eval_documents = lambda r, w: parquet_documents(paths, rank=r, world=w)
        return tok

    def progress(self, elapsed: float) -> float:
        if self.cfg.progress_mode == "steps":
            return min(1.0, self.step_idx / max(1, self.cfg.num_steps))
        return min(1.0, elapsed / max(1e-6, self.cfg.max_train_seconds))

    def train_step(self, elapsed: float = 0.0, read_loss: bool = True) -> float | torch.Tensor:
        cfg = self.cfg
        prog = self.progress(elapsed)
        gas, lr_scale = batch_ramp_grad_accum(cfg, prog, self.grad_accum)
        batches = []
        for _ in range(gas):
            rows = self.loader.next()
            batches.append((rows[:, :-1], rows[:, 1:]))
        update_adamw = (self.step_idx + 1) % cfg.adam_every_n == 0
        model = self.model
        if self.byte_w is not None:
            # byte-weighted loss: route through the model with per-token weights
            orig = model.forward

            def fwd(x, y, _orig=orig):
                return _orig(x, y, row_weight=self.byte_w[y.reshape(-1).long()].contiguous())
            model.forward = fwd
        try:
            loss = self.engine.forward_backward(batches, loss_scale=self.loss_scale,
                                                zero_adamw=self._adamw_applied_last)
        finally:
            if self.byte_w is not None:
                model.forward = orig
        skip = False
        if cfg.loss_scale_dynamic:
            finite = grads_finite_(model, self.engine.layout.grad)
            ov = torch.tensor([0.0 if finite else 1.0], device=self.device)
            if dist.is_available() and dist.is_initialized():
                dist.all_reduce(ov, op=dist.ReduceOp.MAX)
            self.loss_scale, self.loss_scale_clean, skip = next_loss_scale(
                self.loss_scale, self.loss_scale_clean, bool(ov.item() == 0.0),
                cfg.loss_scale_growth_interval, cfg.loss_scale_max)
            if skip:
                self.engine.layout.zero_grad()
        unscale_grads_(model, self.engine.layout.grad, self.loss_scale if not skip else 1.0)
        self.engine.sync_and_clip()
        apply_schedules(cfg, self.opt, self.step_idx, prog, lr_scale)
        if not skip:
            self.engine.optimizer_step(update_adamw)
            self._adamw_applied_last = update_adamw
        self.step_idx += 1
        if read_loss:
            return float(loss.item())
        return loss


def main(argv: list[str] | None = None) -> None:
    run(parse_args(argv))


def run(cfg: RunConfig) -> dict:
    """The training loop of ``main`` for an already-built config; returns the summary."""
    device_type = detect_device_type(cfg.device_type)
    ddp, rank, local_rank, world_size, device = init_runtime(device_type, cfg.seed)
    print0(f"config: {json.dumps(cfg.model_config().__dict__)}")
    tr = Trainer(cfg, device, rank, world_size)
    if cfg.resume_from:
        tr.load_resume(Path(cfg.resume_from) / f"resume_rank{rank}.pt" if Path(cfg.resume_from).is_dir()
                       else cfg.resume_from)
        print0(f"resumed at step {tr.step_idx}")
    nparams = sum(p.numel() for p in tr.model.parameters())
    flops_per_token = tr.model.estimate_flops()
    print0(f"num_params={nparams:,} flops_per_token={flops_per_token:e} grad_accum={tr.grad_accum} "
           f"grad_sync={tr.engine.grad_sync}")
    if cfg.compile_only:
        tr.train_step()
        synchronize(device)
        print0("compile-only synthetic training step completed")
        cleanup_runtime()
        return
    ema_decays = parse_float_tuple(cfg.weight_ema_decay)
    ema_shadows = None
    ema_updates = 0
    loop_started = time.monotonic()
    budget_started = loop_started
    recent: list[float] = []
    smooth = 0.0
    total_tokens = tr.step_idx * tr.tokens_per_step
    step = tr.step_idx
    gc.collect()
    while step < cfg.num_steps:
        elapsed = time.monotonic() - budget_started
        synchronize(device)
        t0 = time.monotonic()
        loss = tr.train_step(elapsed)
        if cfg.weight_ema and tr.progress(elapsed) >= cfg.weight_ema_start_frac:
            with torch.no_grad():
                live = [p for p in tr.model.parameters()]
                if ema_shadows is None:
                    ema_shadows = [[p.detach().clone() for p in live] for _ in ema_decays]
                else:
                    for sh, d in zip(ema_shadows, ema_decays):
                        torch._foreach_lerp_(sh, live, 1.0 - d)
                    ema_updates += 1
        synchronize(device)
        record_step_boundary(step)
        dt = time.monotonic() - t0
        recent.append(dt)
        if step + 1 == TRAIN_STARTUP_STEPS_EXCLUDED:
            budget_started = time.monotonic()
        el2 = time.monotonic() - budget_started
        reached = step + 1 >= TRAIN_STARTUP_STEPS_EXCLUDED
        cap_hit = step + 1 >= cfg.num_steps
        time_hit = cfg.progress_mode == "time" and reached and (
            el2 >= cfg.max_train_seconds or el2 + max(recent[-20:]) + 15.0 >= cfg.max_train_seconds)
        control = torch.tensor([1 if (math.isnan(loss) or loss > 100) else 0, 1 if (cap_hit or time_hit) else 0],
                               device=device, dtype=torch.int32)
        if ddp:
            dist.all_reduce(control, op=dist.ReduceOp.MAX)
        if int(control[0].item()):
            raise RuntimeError(f"bad loss detected: {loss}")
        total_tokens += tr.tokens_per_step
        if step == 0:
            gc.collect()
            gc.freeze()   # long-lived objects out of the collector's way after the first step
        smooth = 0.9 * smooth + 0.1 * loss
        deb = smooth / (1 - 0.9 ** (step + 1))
        if step < 5 or step % cfg.log_every == 0:
            print0(f"step {step:05d} | loss {deb:.4f} | dt {dt:.3f}s | tok/s {tr.tokens_per_step / max(dt, 1e-9):,.0f} "
                   f"| mfu {flops_per_token * tr.tokens_per_step / max(dt, 1e-9) / 1e12:.0f} TF/s", flush=True)
        step += 1
        if cfg.save_every > 0 and step % cfg.save_every == 0:
            tr.save_resume(Path(cfg.out_dir) / "resume" / f"resume_rank{rank}.pt")
        if int(control[1].item()):
            break
    out = Path(cfg.out_dir) / "final.pt"
    if rank == 0:
        ema_state = None
        if ema_shadows is not None:
            state = dict(tr.model.state_dict())
            names = [n for n, _ in tr.model.named_parameters()]
            for n, t in zip(names, ema_shadows[0]):
                state[n] = t
            ema_state = state
        ckpt.save_checkpoint(out, tr.model, {"step": step, "total_train_tokens": total_tokens,
                                              "world_size": world_size, "weight_ema_updates": ema_updates},
                             ema_state=ema_state)
    if ddp:
        dist.barrier()
    if cfg.eval_public:
        tr.model.disable_tp()
        tok = tr.eval_tokenizer()
        causal = causality_check(tr.model, tok, cfg.device_batch_size, cfg.seq_len, device)
        rows = max(1, cfg.device_batch_size * cfg.pack_factor)
        res = evaluate_bpb(tr.model, tok, rows, cfg.seq_len, device, max_tokens=cfg.eval_tokens)
        extra = {}
        if cfg.eval_seq_len > 0 and cfg.eval_seq_len != cfg.seq_len:
            alt = evaluate_bpb(tr.model, tok, rows, cfg.eval_seq_len, device, max_tokens=cfg.eval_tokens)
            extra.update(eval_alt_seq_len=cfg.eval_seq_len, val_bpb_alt=alt["val_bpb"], eval_alt_seconds=alt["eval_seconds"])
        if ema_shadows is not None:
            live = [p.detach().clone() for p in tr.model.parameters()]
            with torch.no_grad():
                for p, e in zip(tr.model.parameters(), ema_shadows[0]):
                    p.copy_(e)
            tr.engine.layout.refresh_bf16()
            ema = evaluate_bpb(tr.model, tok, rows, cfg.seq_len, device, max_tokens=cfg.eval_tokens)
            extra.update(val_bpb_ema=ema["val_bpb"], weight_ema_updates=ema_updates)
            with torch.no_grad():
                for p, v in zip(tr.model.parameters(), live):
                    p.copy_(v)
            tr.engine.layout.refresh_bf16()
        print0("---")
        print0(f"val_bpb: {res['val_bpb']:.6f}")
        print0(f"causality_passed: {causal['passed']}")
        print0(f"causality_max_abs: {causal['max_abs_diff']:.3e}")
        print0(f"eval_tokens: {res['num_tokens']}")
        print0(f"eval_seconds: {res['eval_seconds']:.2f}")
        for k, v in extra.items():
            print0(f"{k}: {v:.6f}" if isinstance(v, float) else f"{k}: {v}")
    print0(f"steps: {step}")
    print0(f"total_train_tokens: {total_tokens}")
    print0(f"num_params: {nparams}")
    summary = {"steps": step, "total_train_tokens": total_tokens, "num_params": nparams}
    if cfg.eval_public:
        summary.update(val_bpb=res["val_bpb"], causality_passed=causal["passed"])
    cleanup_runtime()
    return summary


if __name__ == "__main__":
    main(sys.argv[1:])
