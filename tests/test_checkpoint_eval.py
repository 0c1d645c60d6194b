"""out/final.pt layout, load_for_eval / warm start contracts, evaluate_bpb, causality."""
import math

import torch

from _refutil import build_reference_tiny, import_reference
from trainium_frontier_b200 import checkpoint as ckpt
from trainium_frontier_b200.config import preset
from trainium_frontier_b200.data.synthetic import SyntheticTokenizer
from trainium_frontier_b200.eval import causality_check, evaluate_bpb
from trainium_frontier_b200.models.gpt import GPT


def _tiny():
    cfg = preset("tiny")
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    return cfg, m


def test_final_pt_layout_and_load_for_eval(tmp_path):
    cfg, m = _tiny()
    path = tmp_path / "out" / "final.pt"
    ckpt.save_checkpoint(path, m, {"step": 3, "total_train_tokens": 99})
    payload = torch.load(path, map_location="cpu", weights_only=True)
    assert set(payload) == {"model_state", "model_config", "toggles", "meta"}
    assert payload["model_config"]["n_layer"] == 4 and payload["meta"]["step"] == 3
    ev = ckpt.load_for_eval(str(path), torch.device("cpu"))
    assert ev.config.sequence_len >= 8192 and not ev.training
    for k, v in m.state_dict().items():
        assert torch.equal(ev.state_dict()[k], v), k


def test_ema_state_preferred(tmp_path):
    cfg, m = _tiny()
    ema = {k: torch.zeros_like(v) if v.is_floating_point() else v for k, v in m.state_dict().items()}
    path = tmp_path / "final.pt"
    ckpt.save_checkpoint(path, m, {"step": 1}, ema_state=ema)
    ev = ckpt.load_for_eval(str(path), torch.device("cpu"))
    assert float(ev.transformer.wte.weight.abs().sum()) == 0.0


def test_warm_start(tmp_path):
    cfg, m = _tiny()
    path = tmp_path / "final.pt"
    ckpt.save_checkpoint(path, m, {"step": 7})
    torch.manual_seed(123)
    _, m2 = _tiny()
    meta = ckpt.warm_start_from(str(path), m2)
    assert meta["step"] == 7
    assert torch.equal(m2.lm_head.weight, m.lm_head.weight)


def test_reference_model_loads_our_checkpoint(tmp_path):
    rtrain = import_reference()
    ref = build_reference_tiny(rtrain)
    _, m = _tiny()
    path = tmp_path / "final.pt"
    ckpt.save_checkpoint(path, m, {"step": 0})
    payload = torch.load(path, map_location="cpu", weights_only=True)
    ref.load_state_dict(payload["model_state"], strict=True)


def test_evaluate_bpb_contract_and_value():
    cfg, m = _tiny()
    with torch.no_grad():
        m.lm_head.weight.zero_()  # uniform predictions: CE = ln(8192) per token
    tok = SyntheticTokenizer()
    res = evaluate_bpb(m, tok, 4, 256, "cpu", max_tokens=4096)
    assert set(res) == {"val_bpb", "eval_seconds", "eval_timeout", "eval_over_timeout", "num_tokens",
                        "num_bytes", "total_nats"}
    assert res["num_tokens"] >= 4096
    expected_nats_per_tok = math.log(8192)
    assert abs(res["total_nats"] / res["num_tokens"] - expected_nats_per_tok) < 0.1
    assert res["val_bpb"] > 0


def test_causality_check_passes():
    cfg, m = _tiny()
    res = causality_check(m, SyntheticTokenizer(), 2, 256, "cpu")
    assert res["passed"] and res["max_abs_diff"] <= 1e-5
