"""Trusted harness: the counterpart of the reference's ``prepare.py`` (constants, runtime
helpers, data setup, static submission checks and the ``setup`` / ``check`` /
``eval-public`` CLI).

    python -m trainium_frontier_b200.harness setup
    python -m trainium_frontier_b200.harness check --train-py train.py [--launch-command "torchrun ..."]
    python -m trainium_frontier_b200.harness eval-public --train-py train.py --checkpoint out/final.pt

Differences that follow from the hardware and the offline box:

* ``setup`` materialises the synthetic corpus (the seeded Zipf(1.1) document stream,
  ``data.synthetic``) instead of downloading ClimbMix shards: it writes the per-token
  byte-length table and a manifest of the public train / val stream seeds with their
  SHA-256 digests into the cache directory, so later runs can verify they read the same
  data (the reference verifies its tokenizer artifacts the same way, ``prepare.py:209-225``);
* ``check`` applies the same AST rules as ``prepare.py:690-798`` (forbidden imports and
  calls, a required ``record_step_boundary`` call) and a launch-command rule for one
  process per B200: ``torchrun --nproc-per-node`` (or ``--nproc_per_node``) in {1, 2, 4, 8},
  no shell metacharacters;
* ``eval-public`` imports a training script, calls its ``load_for_eval(path, device)``
  and scores the model with ``eval.evaluate_bpb`` (NCCL / gloo process group when
  launched under torchrun), printing the result dict as JSON on rank 0.
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import importlib.util
import json
import os
import shlex
import sys
from pathlib import Path

import torch
import torch.distributed as dist

from .config import EVAL_TIMEOUT_SECONDS, TOKENIZER_VOCAB_SIZE, TRAIN_STARTUP_STEPS_EXCLUDED
from .runtime import get_dist_info, print0
from .train import record_step_boundary

TRAIN_TIME_BUDGET_SECONDS = 30 * 60
TRAIN_STARTUP_ALLOWANCE_CAP_SECONDS = 900
CACHE_DIR = Path(os.environ.get("NEURON_COMPETITION_R1_CACHE_DIR", Path.home() / ".cache" / "trainium_frontier_b200"))
SPECIAL_TOKENS = [f"<|reserved_{i}|>" for i in range(4)]
BOS_TOKEN = SPECIAL_TOKENS[0]
PUBLIC_SPLITS = ("train", "public_val")
ALLOWED_NPROC = {"1", "2", "4", "8"}

__all__ = ["TRAIN_TIME_BUDGET_SECONDS", "EVAL_TIMEOUT_SECONDS", "TRAIN_STARTUP_STEPS_EXCLUDED",
           "TRAIN_STARTUP_ALLOWANCE_CAP_SECONDS", "TOKENIZER_VOCAB_SIZE", "print0", "get_dist_info",
           "record_step_boundary", "sha256_file", "torch_load_weights", "ensure_data", "check_submission", "main"]


# --------------------------------------------------------------------------- helpers
def sha256_file(path: str | Path, chunk: int = 1 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def torch_load_weights(path: str | Path, map_location):
    return torch.load(path, map_location=map_location, weights_only=True)


# --------------------------------------------------------------------------- setup
def ensure_data(cache_dir: str | Path = CACHE_DIR, stream_tokens: int = 1 << 20, verify: bool = True) -> dict:
    """Write (or verify) the synthetic corpus manifest: byte-length table + digests of the
    first ``stream_tokens`` tokens of every public split's rank-0 stream."""
    from .data import synthetic as syn
    from .data.loader import _packer
    cache = Path(cache_dir)
    cache.mkdir(parents=True, exist_ok=True)
    tb = syn.get_token_bytes("cpu", TOKENIZER_VOCAB_SIZE)
    tb_path = cache / "token_bytes.pt"
    torch.save(tb, tb_path)
    manifest = {"vocab_size": TOKENIZER_VOCAB_SIZE, "bos": syn.BOS_ID, "zipf_s": syn.ZIPF_S,
                "mean_doc_len": syn.MEAN_DOC_LEN, "token_bytes_sha256": hashlib.sha256(tb.numpy().tobytes()).hexdigest(),
                "splits": {}}
    for split in PUBLIC_SPLITS:
        t = torch.empty(stream_tokens, dtype=torch.int32)
        _packer(split, 0).fill_stream(t)
        manifest["splits"][split] = {"tokens": stream_tokens, "sha256": hashlib.sha256(t.numpy().tobytes()).hexdigest()}
    mpath = cache / "manifest.json"
    if verify and mpath.exists():
        old = json.loads(mpath.read_text())
        if old != manifest:
            raise RuntimeError(f"synthetic corpus manifest mismatch in {mpath}: generator or seeds changed")
    mpath.write_text(json.dumps(manifest, indent=1, sort_keys=True))
    return manifest


def ensure_tokenizer(cache_dir: str | Path = CACHE_DIR, archive: str | Path | None = None, **pins):
    """Verify the trusted tokenizer archive (its SHA-256 pins, or ``pins`` overrides:
    ``expected_sha``, ``pkl_sha``, ``token_bytes_sha``, ``expected_vocab``), unpack it into
    ``<cache_dir>/tokenizer`` and return the loaded ``Tokenizer``; None when no archive is
    named.  The training pipeline itself runs on the synthetic corpus.
    Reference counterpart: ``ensure_tokenizer`` (``prepare.py:368-396``)."""
    if not archive:
        return None
    from .data.tokenizer import Tokenizer
    return Tokenizer.from_zip(archive, Path(cache_dir) / "tokenizer", **pins)


# --------------------------------------------------------------------------- static checks
FORBIDDEN_IMPORT_ROOTS = frozenset({"socket", "subprocess", "requests", "urllib", "http", "ftplib"})
FORBIDDEN_ATTR_CALLS = frozenset({("os", "system"), ("os", "popen"), ("shutil", "rmtree"), ("subprocess", "run"),
                                  ("subprocess", "Popen"), ("subprocess", "check_call"),
                                  ("subprocess", "check_output")})
FORBIDDEN_NAME_CALLS = frozenset({"eval", "exec", "__import__", "compile"})


class _Scanner(ast.NodeVisitor):
    def __init__(self):
        self.problems: list[str] = []
        self.step_boundary = False

    def _imp(self, name: str) -> None:
        if name.split(".")[0] in FORBIDDEN_IMPORT_ROOTS:
            self.problems.append(f"forbidden import: {name}")

    def visit_Import(self, node):
        for a in node.names:
            self._imp(a.name)
        self.generic_visit(node)

    def visit_ImportFrom(self, node):
        self._imp(node.module or "")
        self.generic_visit(node)

    def visit_Call(self, node):
        f = node.func
        if isinstance(f, ast.Attribute):
            if f.attr == "record_step_boundary":
                self.step_boundary = True
            if isinstance(f.value, ast.Name) and (f.value.id, f.attr) in FORBIDDEN_ATTR_CALLS:
                self.problems.append(f"forbidden call: {f.value.id}.{f.attr}")
        elif isinstance(f, ast.Name):
            if f.id == "record_step_boundary":
                self.step_boundary = True
            if f.id in FORBIDDEN_NAME_CALLS:
                self.problems.append(f"forbidden call: {f.id}()")
        self.generic_visit(node)


def launch_command_warnings(cmd: str, entrypoint: str) -> list[str]:
    out: list[str] = []
    for tok in ("|", ">", "<", "&&", "||", ";", "&", "`", "$("):
        if tok in cmd:
            out.append(f"launch command contains disallowed shell token: {tok}")
    try:
        toks = shlex.split(cmd)
    except ValueError as e:
        return out + [f"launch command parse error: {e}"]
    i = 0
    while i < len(toks) and "=" in toks[i] and not toks[i].startswith("-"):
        i += 1  # leading VAR=value environment assignments
    if i >= len(toks):
        return out + ["launch command missing executable"]
    exe, args = Path(toks[i]).name, toks[i + 1:]
    if exe not in ("torchrun", "python", "python3"):
        return out + ["launch executable must be torchrun, python, or python3"]
    if exe == "torchrun":
        nproc = None
        for j, a in enumerate(args):
            for flag in ("--nproc-per-node", "--nproc_per_node"):
                if a.startswith(flag + "="):
                    nproc = a.split("=", 1)[1]
                elif a == flag and j + 1 < len(args):
                    nproc = args[j + 1]
        if nproc not in ALLOWED_NPROC:
            out.append("torchrun --nproc-per-node must be 1, 2, 4 or 8 (one process per B200)")
        if not any(Path(a).name == entrypoint for a in args):
            out.append(f"torchrun launch command must target {entrypoint}")
    else:
        script = [a for a in args if not a.startswith("-")]
        if not script or Path(script[0]).name != entrypoint:
            out.append(f"python launch command must target {entrypoint}")
    return out


def check_submission(train_py_path: str, launch_command: str | None = None, *,
                     expected_entrypoint: str | None = None) -> list[str]:
    path = Path(train_py_path)
    sc = _Scanner()
    sc.visit(ast.parse(path.read_text(encoding="utf-8"), filename=str(path)))
    warnings = list(sc.problems)
    if not sc.step_boundary:
        warnings.append("the training script never calls record_step_boundary(); optimizer-step boundaries "
                        "cannot be observed, so the startup allowance cannot be applied")
    if launch_command:
        warnings.extend(launch_command_warnings(launch_command, expected_entrypoint or path.name))
    return warnings


# --------------------------------------------------------------------------- eval-public
def _import_script(path: str):
    p = Path(path).resolve()
    spec = importlib.util.spec_from_file_location("tfb_submission_for_eval", p)
    if spec is None or spec.loader is None:
        raise RuntimeError(f"could not import {p}")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def eval_public(train_py: str, checkpoint: str, device: str = "", batch_size: int = 1, seq_len: int = 1024,
                eval_tokens: int = 4 * 524288, timeout_seconds: int = EVAL_TIMEOUT_SECONDS,
                text_val_data: str = "", tokenizer_zip: str = "", cache_dir: str | Path = CACHE_DIR) -> dict:
    """Scores a checkpoint through the training script's own ``load_for_eval``: on the
    synthetic held-out stream, or with ``text_val_data`` (parquet glob) on held-out text
    tokenized with the verified ``tokenizer_zip``."""
    from .data.synthetic import SyntheticTokenizer
    from .eval import evaluate_bpb
    tok = SyntheticTokenizer(TOKENIZER_VOCAB_SIZE)
    if text_val_data:
        import glob
        from .data.text_loader import parquet_documents
        # the model's vocabulary is checked against the tokenizer's by evaluate_bpb itself
        tok = ensure_tokenizer(cache_dir, tokenizer_zip, expected_vocab=None)
        if tok is None:
            raise RuntimeError("held-out text needs --tokenizer-zip")
        paths = sorted(glob.glob(text_val_data))
        if not paths:
            raise RuntimeError(f"{text_val_data!r} matches no files")
        tok.eval_documents = lambda r, w: parquet_documents(paths, rank=r, world=w)
    mod = _import_script(train_py)
    if not hasattr(mod, "load_for_eval"):
        raise RuntimeError("the training script must define load_for_eval(checkpoint_path, device)")
    dev = torch.device(device) if device else torch.device("cuda" if torch.cuda.is_available() else "cpu")
    ddp, _rank, local, _world = get_dist_info()
    own_pg = False
    if ddp and not (dist.is_available() and dist.is_initialized()):
        if dev.type == "cuda":
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            dist.init_process_group("nccl", device_id=dev)
        else:
            dist.init_process_group("gloo")
        own_pg = True
    try:
        model = mod.load_for_eval(checkpoint, dev)
        return evaluate_bpb(model, tok, batch_size, seq_len, dev,
                            split="public_val", max_tokens=None if eval_tokens <= 0 else eval_tokens,
                            timeout_seconds=timeout_seconds)
    finally:
        if own_pg:
            dist.destroy_process_group()


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description="trainium_frontier_b200 harness")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("setup")
    s.add_argument("--cache-dir", default=str(CACHE_DIR))
    s.add_argument("--stream-tokens", type=int, default=1 << 20)
    s.add_argument("--tokenizer-zip", default=os.environ.get("NEURON_COMPETITION_R1_TOKENIZER_PATH", ""),
                   help="trusted 8192-token tokenizer archive to verify and unpack (optional)")
    c = sub.add_parser("check")
    c.add_argument("--train-py", required=True)
    c.add_argument("--launch-command", default=None)
    e = sub.add_parser("eval-public")
    e.add_argument("--train-py", required=True)
    e.add_argument("--checkpoint", required=True)
    e.add_argument("--device", default="")
    e.add_argument("--batch-size", type=int, default=1)
    e.add_argument("--seq-len", type=int, default=1024)
    e.add_argument("--eval-tokens", type=int, default=4 * 524288, help="0 = the whole public stream")
    e.add_argument("--timeout-seconds", type=int, default=EVAL_TIMEOUT_SECONDS)
    e.add_argument("--text-val-data", default="", help="glob of held-out parquet text (default: synthetic stream)")
    e.add_argument("--tokenizer-zip", default=os.environ.get("NEURON_COMPETITION_R1_TOKENIZER_PATH", ""))
    e.add_argument("--cache-dir", default=str(CACHE_DIR))
    a = ap.parse_args(argv)
    if a.cmd == "setup":
        m = ensure_data(a.cache_dir, a.stream_tokens)
        tok = ensure_tokenizer(a.cache_dir, a.tokenizer_zip)
        if tok is not None:
            print(f"tokenizer verified: vocab {tok.get_vocab_size()}, BOS {tok.get_bos_token_id()}")
        print(f"setup complete: {a.cache_dir} (token bytes {m['token_bytes_sha256'][:12]}...)")
    elif a.cmd == "check":
        w = check_submission(a.train_py, a.launch_command)
        if w:
            for x in w:
                print(f"WARNING: {x}")
            raise SystemExit(1)
        print("check passed")
    else:
        res = eval_public(a.train_py, a.checkpoint, a.device, a.batch_size, a.seq_len, a.eval_tokens, a.timeout_seconds,
                          a.text_val_data, a.tokenizer_zip, a.cache_dir)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(res, indent=2, sort_keys=True))


if __name__ == "__main__":
    main()
