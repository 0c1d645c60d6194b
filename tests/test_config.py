"""Flag / env configuration system."""
import pytest

from trainium_frontier_b200.config import RunConfig, parse_args, preset


def test_width_derivation_matches_reference_rule():
    g = RunConfig(depth=6, aspect_ratio=96, head_dim=128).model_config()
    assert (g.n_embd, g.n_head, g.n_layer) == (640, 5, 6)
    g = preset("d20").model_config()
    assert (g.n_embd, g.n_head, g.head_dim) == (1280, 10, 128)


def test_env_override_then_cli_override(monkeypatch):
    monkeypatch.setenv("NEURON_COMPETITION_R1_DEPTH", "8")
    monkeypatch.setenv("NEURON_COMPETITION_R1_VE", "1")
    cfg = parse_args([])
    assert cfg.depth == 8 and cfg.ve is True
    cfg = parse_args(["--depth", "3", "--no-ve"])
    assert cfg.depth == 3 and cfg.ve is False


def test_validation():
    with pytest.raises(ValueError):
        parse_args(["--clip-order", "sideways"])
    with pytest.raises(ValueError):
        RunConfig(n_embd=100, head_dim=64).model_config()
    with pytest.raises(ValueError):
        RunConfig(depth=6, n_kv_heads=3).model_config()


def test_reference_only_flags_parse():
    """Launch commands written for the reference carry switches whose effect this
    framework always has; they parse, and the ones with an effect here map to it."""
    from trainium_frontier_b200.config import ACCEPTED_NO_EFFECT_FLAGS
    argv = []
    for flag in ACCEPTED_NO_EFFECT_FLAGS:
        argv.append(flag)
    argv += ["--no-nki-muon", "--grad-bucket", "--no-transposed-linear", "--epoch-shuffle",
             "--epoch-shuffle-seed", "77", "--attn-cproj-init", "0.25", "--no-out-bigram-bf16",
             "--coalesced-swiglu-hidden", "256"]
    cfg = parse_args(argv)
    assert cfg.grad_sync == "bucket"
    assert cfg.epoch_shuffle and cfg.epoch_shuffle_seed == 77
    assert cfg.attn_cproj_init_scale == 0.25 and cfg.out_bigram_bf16 is False
    assert cfg.coalesced_swiglu_hidden == 256
    with pytest.raises(ValueError, match="transposed-linear"):
        parse_args(["--transposed-linear"])
    with pytest.raises(ValueError):
        parse_args(["--coalesced-swiglu-hidden", "100"])


def test_coalesced_swiglu_hidden_and_bigram_dtype_shape_the_model():
    import torch
    from trainium_frontier_b200.models.gpt import GPT
    rc = preset("tiny", depth=2, coalesced_swiglu=True, coalesced_swiglu_hidden=384, out_bigram=True)
    m = GPT(rc.model_config(), rc)
    assert m.transformer.h[0].mlp.c_fc.weight.shape == (2 * 384, 256)
    assert m.out_bigram.weight.dtype == torch.bfloat16
    rc2 = rc.replace(out_bigram_bf16=False)
    assert GPT(rc2.model_config(), rc2).out_bigram.weight.dtype == torch.float32
