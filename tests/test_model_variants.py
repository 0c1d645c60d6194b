"""Optional members of the model family on the CPU oracle path: every variant is an exact
no-op at initialisation (same loss as the plain model carrying the same shared weights),
and trains (finite, decreasing loss)."""
import pytest
import torch

VARIANTS = {
    "engram": dict(engram=True, engram_site="1", engram_table_mult=2, engram_mem_dim=32),
    "engram_keydim": dict(engram=True, engram_site="-1", engram_table_mult=2, engram_mem_dim=32, engram_key_dim=64,
                          engram_orders="2", engram_heads=2, engram_conv_kernel=0),
    "engram_share": dict(engram=True, engram_site="1", engram_share_ngram_tables=True, ngram_ve=True,
                         ngram_ve_layers="0,1", ngram_ve_table_mult=2),
    "parallel_block": dict(parallel_block=True),
    "block_nudge_qk": dict(block_nudge=True, block_nudge_site="qk"),
    "block_nudge_resid": dict(block_nudge=True, block_nudge_site="resid"),
    "selective_gate": dict(selective_gate=True, selective_gate_channels=16),
}


def _model(**kw):
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.models.gpt import GPT
    cfg = preset("tiny", depth=3, **kw)
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    return cfg, m


def _batch():
    g = torch.Generator().manual_seed(3)
    x = torch.randint(1, 8192, (2, 129), generator=g)
    return x[:, :-1], x[:, 1:]


@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_variant_is_noop_at_init(name):
    _, base = _model()
    kw = VARIANTS[name]
    _, var = _model(**kw)
    if kw.get("ngram_ve"):
        _, base = _model(ngram_ve=True, ngram_ve_layers=kw["ngram_ve_layers"], ngram_ve_table_mult=2)
    shared = {k: v for k, v in base.state_dict().items() if k in var.state_dict()}
    missing = var.load_state_dict(shared, strict=False)
    assert not missing.unexpected_keys
    x, y = _batch()
    with torch.no_grad():
        a, b = float(base(x, y)), float(var(x, y))
    assert abs(a - b) < 1e-5, (name, a, b)


@pytest.mark.parametrize("name", ["engram", "parallel_block", "selective_gate", "block_nudge_qk"])
def test_variant_trains(name):
    from trainium_frontier_b200.engine import TrainEngine
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    cfg, m = _model(**VARIANTS[name])
    opt = setup_optimizer(m, cfg, torch.float32)
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 1, "none")
    x, y = _batch()
    losses = []
    for _ in range(4):
        losses.append(float(eng.forward_backward([(x, y)])))
        eng.sync_and_clip()
        eng.optimizer_step()
    assert all(l == l for l in losses) and losses[-1] < losses[0], losses
    if name == "block_nudge_qk":
        assert all(float(b.block_nudge.abs().sum()) == 0.0 for b in m.transformer.h)


def test_qkv_attention_entry_matches_composition():
    """ops.qkv_attention (projection + RoPE + QK-norm + attention from the block input)
    equals the projection followed by attention_qkv on the CPU oracle path."""
    from trainium_frontier_b200 import ops
    torch.manual_seed(5)
    B, T, H, D = 2, 128, 2, 64
    C = H * D
    t = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    tab = torch.outer(t, inv)
    cos, sin = tab.cos()[None, :, None, :], tab.sin()[None, :, None, :]
    x = torch.randn(B, T, C)
    ws = [torch.randn(C, C) * C ** -0.5 for _ in range(3)]
    a = ops.qkv_attention(x, ws, cos, sin, H, D, None)
    b = ops.attention_qkv(ops.linear_multi(x, ws), cos, sin, H, D, None)
    assert a.shape == (B, T, C) and torch.allclose(a, b)
