"""Inference / evaluation benchmark of a random-init d20 checkpoint in the out/final.pt layout.

Two workloads, both through the public API (``checkpoint.load_for_eval``):

* held-out evaluation: forward-only loss and bpb over 2^20 synthetic Zipf tokens at seq
  2048 (rows of 32 sequences, data parallel across ranks, the per-rank token cap of the
  trusted harness).  ``value`` = tokens / device time of the forward + fp32 CE over
  device-resident rows (CUDA events, max over ranks); ``e2e`` = the trusted harness
  ``evaluate_bpb`` itself (host-built rows, pinned H2D copies, scalar reads), wall clock,
  max over ranks.
* KV-cache greedy decode: 256 new tokens for a batch of 32 sequences with 512-token
  seeded Zipf prompts (the batch split over ranks): prefill through the training kernels,
  then one CUDA-graph replay per token.  Reported as generated tokens / s (all ranks) and
  ms per decode step (max over ranks).

The reference arm loads the same checkpoint with the reference's own ``load_for_eval`` and
scores it with its own ``evaluate_bpb`` (its loader and byte table pointed at the same
synthetic stream); the reference has no generation path, so its decode entry says so.

Reference counterparts: ``load_for_eval`` (``train.py:4706-4743``) and ``evaluate_bpb``
(``prepare.py:595-659``).
"""
from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

EVAL_TOKENS = 1 << 20
SEQ = 2048
EVAL_ROWS = 32
DEC_BATCH, DEC_PROMPT, DEC_NEW = 32, 512, 256
METRIC = "inference: held-out eval tok/s over 2^20 tokens at seq 2048 (max over ranks); KV-cache greedy decode tok/s (batch 32, 512 prompt + 256 new)"


def _ckpt_path(root: str) -> str:
    return os.path.join(root, "out", "bench_d20", "final.pt")


def ensure_checkpoint(root: str, rank: int) -> str:
    """Rank 0 writes a random-init d20 checkpoint (seed 1234) if none exists."""
    path = _ckpt_path(root)
    if rank == 0 and not os.path.exists(path):
        from ..checkpoint import save_checkpoint
        from ..config import preset
        from ..models.gpt import GPT
        cfg = preset("d20", seed=1234)
        torch.manual_seed(cfg.seed)
        m = GPT(cfg.model_config(), cfg)
        m.init_weights()
        save_checkpoint(path, m, {"step": 0, "total_train_tokens": 0, "note": "random init"})
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    return path


def _staged_rows(dev, rank: int, world: int):
    from ..data.loader import make_eval_dataloader
    from ..data.synthetic import SyntheticTokenizer
    per_rank = -(-EVAL_TOKENS // world)
    out, n = [], 0
    for x, y, _ in make_eval_dataloader(SyntheticTokenizer(8192), EVAL_ROWS, SEQ, "public_val", dev,
                                        max_stream_tokens=EVAL_TOKENS + world * (SEQ + 1)):
        out.append((x, y))
        n += int((y >= 0).sum())
        if n >= per_rank:
            break
    return out


def _device_eval(model, batches, dev, token_bytes):
    nats = torch.zeros((), dtype=torch.float32, device=dev)
    ntok = 0
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        for x, y in batches[:1]:   # warm-up (kernel setup / compile)
            model(x)
        torch.cuda.synchronize(dev)
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
        a.record()
        for x, y in batches:
            logits = model(x)[..., :8192].float()
            loss = F.cross_entropy(logits.reshape(-1, 8192), y.reshape(-1), ignore_index=-1, reduction="none")
            yf = y.reshape(-1)
            nats += (loss * ((yf >= 0) & (token_bytes[yf.clamp_min(0)] > 0))).sum()
        b.record()
        torch.cuda.synchronize(dev)
    for _, y in batches:
        ntok += int((y >= 0).sum())
    return a.elapsed_time(b), ntok, float(nats)


def _max(x: float, dev) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum(x: float, dev) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return float(t.item())


def run(args, impl: str, root: str, rank: int, world: int, local: int, dev) -> dict:
    from ..data import synthetic as syn
    path = ensure_checkpoint(root, rank)
    token_bytes = syn.get_token_bytes(dev, 8192)
    if impl == "ours":
        from ..checkpoint import load_for_eval
        from ..eval import evaluate_bpb
        model = load_for_eval(path, dev)
        harness = evaluate_bpb
    else:
        import sys
        ref_dir = os.path.join(root, "baseline", "_ref")
        sys.path.insert(0, ref_dir)
        saved = sys.argv
        sys.argv = ["train.py"]
        import prepare as rprep  # noqa: E402
        import train as rtrain  # noqa: E402
        sys.argv = saved
        from ..data.loader import make_eval_dataloader
        rprep.make_eval_dataloader = make_eval_dataloader
        rprep.get_token_bytes = lambda d: syn.get_token_bytes(d, 8192)
        # the checkpoint is the plain family member: the reference's module-level toggles
        # decide which optional modules its GPT builds, so switch its extras off first
        for flag in ("USE_VE", "USE_NGRAM_VE", "USE_LOCAL_CONV", "USE_QK_SHIFT", "USE_ENGRAM", "USE_OUT_BIGRAM",
                     "USE_HEAD_GATE", "USE_OUT_POOL", "USE_X0_GATE", "USE_DOC_MASK"):
            if hasattr(rtrain, flag):
                setattr(rtrain, flag, False)
        model = rtrain.load_for_eval(path, dev)
        harness = rprep.evaluate_bpb
    batches = _staged_rows(dev, rank, world)
    ms, ntok, nats = _device_eval(model, batches, dev, token_bytes)
    ms = _max(ms, dev)
    ntok_all = _sum(ntok, dev)
    # trusted harness, end to end
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    res = harness(model, syn.SyntheticTokenizer(8192), EVAL_ROWS, SEQ, dev, max_tokens=EVAL_TOKENS)
    torch.cuda.synchronize(dev)
    e2e_s = _max(time.perf_counter() - t0, dev)
    out = {
        "metric": METRIC, "value": ntok_all / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "ms_per_pass": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf(1.1) held-out stream); random-init d20 checkpoint in out/final.pt layout",
        "config": {"model": "d20 GPT (20L, d1280, 10x128 heads, relu2 MLP 5120, vocab 8192)",
                   "eval_tokens": EVAL_TOKENS, "seq_len": SEQ, "rows_per_forward": EVAL_ROWS,
                   "parallelism": f"dp{world}", "l2": "inputs larger than L2 (2 GB fp32 logits per forward)"},
        "eval": {"val_bpb": res["val_bpb"], "num_tokens": res["num_tokens"], "device_ms": ms},
        "e2e": {"value": res["num_tokens"] / e2e_s, "unit": "tokens/s", "seconds": e2e_s,
                "api": "evaluate_bpb(load_for_eval(out/final.pt))",
                "h2d_bytes_per_step": EVAL_ROWS * SEQ * (4 + 8), "d2h_bytes_per_step": 8},
        "impl": impl,
    }
    if impl == "ours":
        out["decode"] = _decode(model, dev, rank, world)
    else:
        out["decode"] = {"unavailable": "the reference has no generation / KV-cache path"}
    return out


def _decode(model, dev, rank: int, world: int) -> dict:
    from ..data.loader import make_eval_dataloader
    from ..data.synthetic import SyntheticTokenizer
    from ..inference.generate import Generator
    if DEC_BATCH % world:
        return {"unavailable": f"batch {DEC_BATCH} does not split over {world} ranks"}
    b = DEC_BATCH // world
    x, _, _ = next(make_eval_dataloader(SyntheticTokenizer(8192), DEC_BATCH, DEC_PROMPT, "decode_prompts", "cpu",
                                        max_stream_tokens=DEC_BATCH * (DEC_PROMPT + 1) * world + 1, seed=99))
    prompts = x[rank * b:(rank + 1) * b].pin_memory()
    gen = Generator(model, b, DEC_PROMPT + DEC_NEW + 128)
    gen.generate(prompts.to(dev), 8)   # warm-up: builds and captures the decode graph
    torch.cuda.synchronize(dev)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    toks = gen.generate(prompts.to(dev, non_blocking=True), DEC_NEW)
    e.record()
    host = toks.cpu()
    wall = time.perf_counter() - t0
    ms = _max(a.elapsed_time(e), dev)
    wall = _max(wall, dev)
    return {"tokens_per_s": DEC_BATCH * DEC_NEW / (ms / 1000.0), "ms_total": ms,
            "ms_per_token_step": ms / DEC_NEW, "batch": DEC_BATCH, "prompt": DEC_PROMPT, "new_tokens": DEC_NEW,
            "e2e_tokens_per_s": DEC_BATCH * DEC_NEW / wall, "generated_shape": list(host.shape),
            "note": "device time covers prefill + 256 greedy steps (graph replays); e2e adds the prompt H2D and the token D2H"}


def profile_decode(steps: int = 3) -> dict:
    """KV-cache decode of a random-init d20 model (batch 32, 512-token prompts): after a
    warm-up generate (which captures the step's CUDA graph), ``steps`` graph replays are
    bracketed by cudaProfilerStart / Stop (``ncu --profile-from-start off`` sees only them)
    and timed with CUDA events."""
    from ..config import preset
    from ..inference.generate import Generator
    from ..models.gpt import GPT
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset("d20", seed=1234)
    torch.manual_seed(cfg.seed)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    m = m.to(dev)
    m.set_compute_dtype(torch.bfloat16)
    m.eval()
    g = torch.Generator().manual_seed(5)
    prompts = torch.randint(1, 8192, (DEC_BATCH, DEC_PROMPT), generator=g).to(dev)
    gen = Generator(m, DEC_BATCH, DEC_PROMPT + DEC_NEW + 128)
    gen.generate(prompts, 8)
    gen.replay_steps(8, DEC_PROMPT + 64)   # warm replays at a mid-run cache length
    torch.cuda.synchronize(dev)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.cudart().cudaProfilerStart()
    a.record()
    gen.replay_steps(steps, DEC_PROMPT + 64)
    e.record()
    torch.cuda.synchronize(dev)
    torch.cuda.cudart().cudaProfilerStop()
    ms = a.elapsed_time(e) / steps
    return {"ms_per_step": ms, "batch": DEC_BATCH, "cache_len": DEC_PROMPT + 64, "steps": steps}


if __name__ == "__main__":
    import json
    import sys
    if "--decode-profile" in sys.argv:
        n = int(sys.argv[sys.argv.index("--steps") + 1]) if "--steps" in sys.argv else 3
        print(json.dumps(profile_decode(n)))
