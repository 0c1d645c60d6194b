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
