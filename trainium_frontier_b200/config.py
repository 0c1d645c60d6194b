"""Run configuration: one dataclass, every field settable by ``--flag`` or by the
``NEURON_COMPETITION_R1_<FLAG>`` environment variable.

The reference keeps ~150 module-level constants in ``train.py:199-1052`` and writes
argparse results back into globals (``train.py:4999-5830``, env default pattern at
``train.py:5001-5003``).  Here the same knobs live in one ``RunConfig`` instance that
is passed explicitly; flag names and the env-variable prefix are kept identical so a
launch command or environment written for the reference drives this framework the
same way.  ``GPTConfig`` mirrors ``train.py:1407-1427`` field for field (the
checkpoint's ``model_config`` payload is ``asdict(GPTConfig)``).
"""
from __future__ import annotations

import argparse
import dataclasses
import os
from dataclasses import dataclass, field, fields
from typing import Any

ENV_PREFIX = "NEURON_COMPETITION_R1_"

TOKENIZER_VOCAB_SIZE = 8192
TRAIN_TIME_BUDGET_SECONDS = 30 * 60
EVAL_TIMEOUT_SECONDS = 20 * 60
TRAIN_STARTUP_STEPS_EXCLUDED = 5
TRAIN_STARTUP_ALLOWANCE_CAP_SECONDS = 900
EVAL_MIN_SEQ_LEN = 8192

# Polar-Express (a, b, c) coefficients of the 5 Newton-Schulz iterations
# (train.py:3525-3531 and autoresearch/train.py).  These are published constants of
# the Polar Express method; the optimizer math is defined by them.
POLAR_EXPRESS_COEFFS = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)


@dataclass
class GPTConfig:
    """Model shape; identical field names/defaults to the reference so that
    ``GPTConfig(**payload["model_config"])`` loads either project's checkpoints."""
    sequence_len: int
    vocab_size: int
    n_layer: int
    n_head: int
    n_embd: int
    mlp_ratio: int = 4
    attn_scale: float = 0.0
    n_kv_heads: int = 0

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def padded_vocab_size(self) -> int:
        return ((self.vocab_size + 63) // 64) * 64


def _b(x: str) -> bool:
    return str(x).strip().lower() not in ("0", "false", "no", "off", "")


@dataclass
class RunConfig:
    # ---- shape -------------------------------------------------------------------
    depth: int = 6
    aspect_ratio: int = 96
    head_dim: int = 128
    n_embd: int = 0                 # >0 overrides depth*aspect_ratio rounding
    mlp_ratio: int = 4
    attn_scale: float = 0.0
    n_kv_heads: int = 0
    seq_len: int = 2048
    vocab_size: int = TOKENIZER_VOCAB_SIZE
    rope_base: float = 100000.0
    logit_softcap: float = 15.0
    # ---- batch -------------------------------------------------------------------
    device_batch_size: int = 1
    pack_factor: int = 4
    total_batch_size: int = 131072
    # ---- run control ---------------------------------------------------------------
    num_steps: int = 1_000_000
    max_train_seconds: int = TRAIN_TIME_BUDGET_SECONDS
    progress_mode: str = "time"     # "time" (reference: wall clock) or "steps" (deterministic)
    out_dir: str = "out"
    eval_public: bool = True
    eval_tokens: int = 4 * 524288
    eval_seq_len: int = 0
    device_type: str = ""
    seed: int = 42
    init_from: str = ""
    resume_from: str = ""           # a resume file, or a directory of resume_rank{r}.pt files
    save_every: int = 0             # write <out_dir>/resume/resume_rank{r}.pt every N steps (0 = never)
    compile_only: bool = False
    log_every: int = 10
    # ---- optimizer -----------------------------------------------------------------
    embedding_lr: float = 0.30
    unembedding_lr: float = 0.006
    matrix_lr: float = 0.020
    scalar_lr: float = 0.20
    scalar_beta1: float = 0.9
    scalar_beta2: float = 0.95
    embed_adamw_beta1: float = 0.8
    embed_adamw_beta2: float = 0.95
    lm_head_beta2: float = 0.96
    embedding_wd: float = 0.001
    lm_head_wd: float = 0.01
    weight_decay: float = 0.20
    wd_decay_to_zero: bool = True
    cautious_wd: bool = False
    warmup_steps: int = 0
    warmdown_ratio: float = 0.75
    final_lr_frac: float = 0.05
    lrm_quantum: int = 0
    grad_clip: float = 1.0
    clip_order: str = "local"       # "local" = clip each rank's grads before the average (reference), "global" = after
    muon_ns_steps: int = 5
    muon_beta2: float = 0.90
    muon_beta2_final: float = 0.0
    muon_momentum_warmup_steps: int = 300
    muon_momentum_cooldown_frac: float = 0.045
    muon_momentum_final: float = 0.85
    muon_lr_fp32: bool = False
    muon_depth_lr_bottom: float = 1.0
    muon_depth_lr_top: float = 1.0
    muon_depth_mom_bottom: float = 0.0
    muon_depth_mom_top: float = 0.0
    muon_depth_mom_ref: float = 0.95
    demon_beta1: bool = False
    demon_beta1_final: float = 0.55
    demon_beta1_ref: float = 0.8
    demon_beta1_start_frac: float = -1.0
    adam_every_n: int = 1
    adam_every_n_lr_comp: bool = False
    loss_scale: float = 1.0
    loss_scale_dynamic: bool = False
    loss_scale_growth_interval: int = 500
    loss_scale_max: float = 8192.0
    byte_loss_weight: bool = False
    # ---- init ----------------------------------------------------------------------
    init_scale: float = 0.50
    attn_cproj_init_scale: float = 0.10
    wte_init_std: float = 0.8
    byte_wte_init: bool = False
    byte_wte_init_mix: float = 1.0
    byte_wte_init_ngram: int = 3
    byte_wte_init_std: float = 0.8
    # ---- architecture toggles (all default to the plain family) --------------------
    ve: bool = False
    ve_gate_channels: int = 32
    ve_wd: float = 0.0
    ngram_ve: bool = False
    ngram_ve_layers: str = "1,-1"
    ngram_ve_table_mult: int = 128
    ngram_ve_trigram: bool = True
    ngram_ve_dim: int = 128
    ngram_ve_opt: str = "rmsprop"
    ngram_ve_lr: float = 0.0
    ngram_ve_beta2: float = 0.95
    ngram_ve_flat_lr: bool = True
    ngram_ve_bf16: bool = True
    ngram_ve_clip_exclude: bool = True
    local_conv: bool = False
    local_conv_kernel: int = 2
    train_local_conv: bool = True
    qk_shift: bool = False
    qk_shift_beta: float = 0.0
    qk_shift_freeze: bool = True
    head_gate: bool = False
    head_gate_norm: bool = False
    head_gate_channels: int = 32
    head_gate_bias: float = 0.0
    head_gate_mul: float = 2.0
    out_pool: bool = False
    out_pool_layers: int = 3
    x0_gate: bool = False
    mlp_sandwich_norm: bool = False
    relu2_tau: float = 0.0
    gated_mlp: bool = False
    coalesced_swiglu: bool = False
    coalesced_swiglu_hidden: int = 0   # forced coalesced-SwiGLU hidden width (multiple of 128); 0 = parameter-matched
    parallel_block: bool = False
    doc_mask: bool = False
    window_pattern: str = "L"
    short_window_frac: float = 0.5
    out_bigram: bool = False
    out_bigram_gate_bias: float = -2.0
    out_bigram_lr: float = 0.0
    out_bigram_bf16: bool = True       # store the [V, V] output-bigram table in bf16
    engram: bool = False
    engram_table_mult: int = 32
    engram_mem_dim: int = 128
    engram_conv_kernel: int = 4
    engram_site: str = "2"             # block index after which Y joins the residual (negatives from the end)
    engram_orders: str = "2,3"
    engram_heads: int = 1
    engram_key_dim: int = 0            # 0 -> n_embd (no W_Q)
    engram_share_ngram_tables: bool = False
    engram_bf16: bool = True
    parallel_block_coalesce: str = "none"
    block_nudge: bool = False
    block_nudge_site: str = "qk"       # "qk" or "resid"
    selective_gate: bool = False
    selective_gate_channels: int = 32
    # ---- schedules / extras --------------------------------------------------------
    batch_ramp: bool = False
    batch_ramp_grad_accum: str = "2,4,8"
    batch_ramp_bounds: str = "0.35,0.75"
    batch_ramp_lr_exp: float = 0.5
    weight_ema: bool = False
    weight_ema_decay: str = "0.995"
    weight_ema_start_frac: float = 0.75
    eval_prefer_ema: bool = True
    # ---- B200 engine ----------------------------------------------------------------
    grad_sync: str = "auto"         # auto | per_param | bucket | dist_muon | fused
    bucket_layers: int = 4          # transformer blocks per gradient bucket
    use_cuda_graphs: bool = False
    tp: int = 1                     # tensor-parallel degree (DP = world / tp)
    pp: int = 1                     # pipeline stages (DP = world / pp); tp and pp are exclusive
    checkpoint_activations: bool = False
    # ---- data ----------------------------------------------------------------------
    synthetic_epoch_tokens: int = 0    # tokens per epoch of the synthetic train stream per rank; 0 = endless
    epoch_shuffle: bool = False        # from epoch 2 on, a fresh order (seed + epoch) instead of epoch 1 replayed
    epoch_shuffle_seed: int = 1234
    text_data: str = ""                # glob of parquet files with a "text" column: train on them instead
    tokenizer_zip: str = ""            # the tokenizer archive the text is tokenized with (SHA-verified)
    text_val_data: str = ""            # glob of held-out parquet files the final evaluation scores (with --text-data)
    # ---- reference switches with a real effect here --------------------------------
    grad_bucket: bool = False          # one flat-buffer gradient all-reduce: maps to grad_sync=bucket under auto
    transposed_linear: bool = False    # [in, out] weight storage: not built (changes the checkpoint layout)

    # ------------------------------------------------------------------------------
    def model_config(self) -> GPTConfig:
        """``build_config`` (train.py:3488-3519): width = round_up(depth*aspect, head_dim)
        unless ``n_embd`` is given."""
        if self.n_embd > 0:
            n_embd = self.n_embd
            if n_embd % self.head_dim:
                raise ValueError(f"n_embd={n_embd} must be a multiple of head_dim={self.head_dim}")
        else:
            base = self.depth * self.aspect_ratio
            n_embd = ((base + self.head_dim - 1) // self.head_dim) * self.head_dim
        n_head = n_embd // self.head_dim
        if self.n_kv_heads < 0 or self.n_kv_heads > n_head:
            raise ValueError(f"n_kv_heads={self.n_kv_heads} must be 0 or in [1, {n_head}]")
        if self.n_kv_heads and n_head % self.n_kv_heads:
            raise ValueError(f"n_kv_heads={self.n_kv_heads} must divide n_head={n_head}")
        return GPTConfig(sequence_len=self.seq_len, vocab_size=self.vocab_size, n_layer=self.depth,
                         n_head=n_head, n_embd=n_embd, mlp_ratio=self.mlp_ratio,
                         attn_scale=self.attn_scale, n_kv_heads=self.n_kv_heads)

    def toggles(self) -> dict[str, Any]:
        return {k: getattr(self, k) for k in ARCH_TOGGLE_NAMES}

    def replace(self, **kw) -> "RunConfig":
        return dataclasses.replace(self, **kw)


# Toggles snapshotted into checkpoints (train.py:4533-4664 keeps the same two tiers:
# shape-critical ones change parameter shapes, the rest change behaviour silently).
SHAPE_CRITICAL_TOGGLES = (
    "ve", "ngram_ve", "ngram_ve_layers", "ngram_ve_table_mult", "ngram_ve_trigram",
    "ngram_ve_dim", "ngram_ve_bf16", "local_conv", "local_conv_kernel", "qk_shift",
    "head_gate", "out_pool", "out_pool_layers", "x0_gate", "gated_mlp", "coalesced_swiglu",
    "coalesced_swiglu_hidden", "parallel_block", "out_bigram", "engram", "engram_table_mult", "engram_mem_dim",
    "engram_conv_kernel", "engram_site", "engram_orders", "engram_heads", "engram_key_dim",
    "engram_share_ngram_tables", "engram_bf16", "parallel_block_coalesce", "block_nudge", "block_nudge_site",
    "selective_gate", "selective_gate_channels",
)
ARCH_TOGGLE_NAMES = SHAPE_CRITICAL_TOGGLES + (
    "rope_base", "logit_softcap", "ve_gate_channels", "qk_shift_beta", "qk_shift_freeze",
    "head_gate_norm", "head_gate_channels", "head_gate_bias", "head_gate_mul",
    "mlp_sandwich_norm", "relu2_tau", "doc_mask", "window_pattern", "short_window_frac",
    "out_bigram_gate_bias", "out_bigram_bf16",
)


def _env_default(name: str, default: Any) -> Any:
    key = ENV_PREFIX + name.upper()
    if key not in os.environ:
        return default
    raw = os.environ[key]
    if isinstance(default, bool):
        return _b(raw)
    return type(default)(raw)


def build_parser(base: RunConfig | None = None) -> argparse.ArgumentParser:
    """argparse with one ``--kebab-case`` flag per field; env overrides the default,
    the command line overrides both (same precedence as ``_hp`` at train.py:5168-5170)."""
    base = base or RunConfig()
    p = argparse.ArgumentParser(description="B200 GPT pretraining (trainium_frontier capabilities)")
    for f in fields(RunConfig):
        default = _env_default(f.name, getattr(base, f.name))
        flag = "--" + f.name.replace("_", "-")
        if isinstance(default, bool):
            p.add_argument(flag, dest=f.name, action=argparse.BooleanOptionalAction, default=default)
        else:
            p.add_argument(flag, dest=f.name, type=type(default), default=default)
    # reference-compatible aliases
    p.add_argument("--compile", dest="_compile", action=argparse.BooleanOptionalAction, default=False,
                   help="accepted for launch-command compatibility; the B200 path has no tracing compiler")
    p.add_argument("--attn-cproj-init", dest="attn_cproj_init_scale", type=float,
                   default=_env_default("attn_cproj_init", getattr(base, "attn_cproj_init_scale")),
                   help="the reference's name of --attn-cproj-init-scale")
    # Reference switches (train.py:5014-5110, :5341, :5470) whose effect this framework
    # always has on CUDA, so they are accepted and change nothing:
    for flag, why in ACCEPTED_NO_EFFECT_FLAGS.items():
        p.add_argument(flag, dest="_ref_" + flag[2:].replace("-", "_"), action=argparse.BooleanOptionalAction,
                       default=None, help="accepted; no effect here: " + why)
    return p


# Reference flags accepted for launch-command compatibility, each with why it has no
# effect on this framework's path.
ACCEPTED_NO_EFFECT_FLAGS = {
    "--compile-muon": "Muon's math always runs as fused sm_100a kernels (no tracing compiler)",
    "--foreach-optim": "AdamW is always one multi-tensor launch per group",
    "--clip-foreach": "the clip norm is one fused reduction over the flat gradient buffer",
    "--tensor-lr-scalars": "learning rates and decays always live in device scalars",
    "--nki-relu2": "relu^2 always runs in the MLP GEMM's epilogue on CUDA",
    "--nki-rope-norm": "RoPE + QK-norm always runs fused (QKV GEMM epilogue or its own kernel) on CUDA",
    "--nki-softcap-ce": "softcap + cross-entropy always runs as the fused kernel on CUDA",
    "--nki-muon": "Muon's elementwise steps always run in GEMM epilogues / fused kernels on CUDA",
    "--qkv-norm-cse": "the fused QKV projection normalises its input once by construction",
}


def parse_args(argv: list[str] | None = None, base: RunConfig | None = None) -> RunConfig:
    ns = build_parser(base).parse_args(argv)
    kw = {f.name: getattr(ns, f.name) for f in fields(RunConfig)}
    if kw["grad_bucket"] and kw["grad_sync"] == "auto":
        kw["grad_sync"] = "bucket"
    cfg = RunConfig(**kw)
    validate(cfg)
    return cfg


def validate(cfg: RunConfig) -> None:
    """Cross-flag validation (train.py:5599-5830 does the same class of checks)."""
    if cfg.clip_order not in ("local", "global"):
        raise ValueError("--clip-order must be 'local' or 'global'")
    if cfg.progress_mode not in ("time", "steps"):
        raise ValueError("--progress-mode must be 'time' or 'steps'")
    if cfg.grad_sync not in ("auto", "per_param", "bucket", "dist_muon", "fused"):
        raise ValueError(f"unknown --grad-sync {cfg.grad_sync}")
    if cfg.transposed_linear:
        raise ValueError("--transposed-linear ([in, out] weight storage) is not built: the tcgen05 GEMM reads "
                         "[out, in] weights K-major in place, and the flag would change every Linear's "
                         "state_dict shape; use --no-transposed-linear (the reference's default)")
    if cfg.coalesced_swiglu_hidden % 128 or cfg.coalesced_swiglu_hidden < 0:
        raise ValueError("--coalesced-swiglu-hidden must be 0 (auto) or a positive multiple of 128")
    if cfg.synthetic_epoch_tokens < 0:
        raise ValueError("--synthetic-epoch-tokens must be >= 0")
    if cfg.coalesced_swiglu and cfg.gated_mlp:
        raise ValueError("--coalesced-swiglu and --gated-mlp are mutually exclusive")
    if cfg.adam_every_n < 1:
        raise ValueError("--adam-every-n must be >= 1")
    if cfg.tp < 1 or cfg.pp < 1:
        raise ValueError("--tp and --pp must be >= 1")
    if cfg.tp > 1 and cfg.pp > 1:
        raise ValueError("--tp and --pp cannot be combined")
    if cfg.parallel_block_coalesce != "none":
        raise ValueError("--parallel-block-coalesce: only 'none' is built (the fused QKV GEMM already reads "
                         "the three attention inputs as one weight); 'vfc' / 'all' change the state_dict layout")
    if cfg.block_nudge_site not in ("qk", "resid"):
        raise ValueError("--block-nudge-site must be 'qk' or 'resid'")
    if cfg.engram:
        orders = [int(o) for o in cfg.engram_orders.split(",") if o.strip()]
        if not orders or any(o not in (2, 3) for o in orders):
            raise ValueError("--engram-orders supports 2 and 3")
    if cfg.ve_gate_channels * 3 > max(cfg.model_config().n_embd, 1) and cfg.ngram_ve:
        raise ValueError("n_embd too small for three value-embedding gate slices")


def parse_float_tuple(s: str) -> tuple[float, ...]:
    return tuple(float(x) for x in str(s).split(",") if x.strip())


def parse_int_tuple(s: str) -> tuple[int, ...]:
    return tuple(int(x) for x in str(s).split(",") if x.strip())


# Named workload presets: the plain-family shapes this framework is benchmarked on.
PRESETS: dict[str, dict[str, Any]] = {
    "tiny": dict(depth=4, n_embd=256, head_dim=64, seq_len=256, rope_base=10000.0,
                 device_batch_size=8, pack_factor=1, total_batch_size=8 * 256),
    "d12": dict(depth=12, n_embd=768, head_dim=128, seq_len=2048, total_batch_size=524288),
    "d20": dict(depth=20, n_embd=1280, head_dim=128, seq_len=2048, total_batch_size=524288),
    "d26": dict(depth=26, n_embd=1664, head_dim=128, seq_len=4096, total_batch_size=1048576),
    # the 5-minute single-GPU research loop (depth 6, aspect 96 -> width 576 rounded up to
    # the 128 head dim; its own learning rates, softcap and rotary base)
    "autoresearch": dict(depth=6, n_embd=640, head_dim=128, seq_len=2048, device_batch_size=16, pack_factor=1,
                         total_batch_size=131072, logit_softcap=11.0, rope_base=2_000_000.0, embedding_lr=0.2,
                         unembedding_lr=0.004, matrix_lr=0.04, scalar_lr=0.3, weight_decay=0.0,
                         embed_adamw_beta1=0.75, embed_adamw_beta2=0.99, warmdown_ratio=0.0, final_lr_frac=0.02,
                         max_train_seconds=300, progress_mode="time", ve=False, ngram_ve=False,
                         local_conv=False, qk_shift=False),
}


def preset(name: str, **overrides) -> RunConfig:
    kw = dict(PRESETS[name])
    kw.update(overrides)
    return RunConfig(**kw)
