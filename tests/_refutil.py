"""Import helper for the reference implementation (installed under baseline/_ref).

The reference's ``train.py`` is imported as a module, the way its own equivalence
harnesses do (argv neutralised), and configured through its module globals.
"""
from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    if not os.path.exists(os.path.join(REF_DIR, "train.py")):
        pytest.skip("reference not installed under baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    argv = sys.argv
    sys.argv = ["train.py"]
    try:
        import train as rtrain  # noqa: E402
    finally:
        sys.argv = argv
    return rtrain


def configure_tiny(rtrain):
    """The plain tiny member: 4 layers, d256, 4 x 64 heads, seq 256, RoPE base 10000."""
    rtrain.DEPTH = 4
    rtrain.N_EMBD = 256
    rtrain.HEAD_DIM = 64
    rtrain.SEQ_LEN = 256
    rtrain.USE_VE = False
    rtrain.USE_NGRAM_VE = False
    rtrain.USE_LOCAL_CONV = False
    rtrain.USE_QK_SHIFT = False
    rtrain.COMPUTE_DTYPE = torch.float32
    rtrain.TOKENIZER_VOCAB_SIZE = 8192


def build_reference_tiny(rtrain, seed: int = 0):
    configure_tiny(rtrain)
    torch.manual_seed(seed)
    cfg = rtrain.build_config()
    model = rtrain.GPT(cfg)
    model.init_weights()
    cos, sin = model._precompute_rotary_embeddings(cfg.sequence_len, cfg.n_embd // cfg.n_head, base=10000)
    model.cos.copy_(cos)
    model.sin.copy_(sin)
    return model
