"""Loss parity against the reference's own train.py on CPU (fp32), tiny plain config.

Both models start from the same weights (the reference's init, loaded into ours by
state_dict -- the key layout is shared) and see the same synthetic batches; both
optimizers get the same per-step lr / momentum / weight-decay schedule.  ws=1 here;
the gloo ws=2 variant is ``test_dist_cpu.py::test_loss_parity_with_reference_ws2``.
After training, both models are scored by the same ``evaluate_bpb`` on the same held-out
tokens (parity of held-out bpb at equal training tokens).
"""
import math

import pytest
import torch

from _refutil import build_reference_tiny, import_reference


def _batches(n, B=8, T=256, seed=11):
    from trainium_frontier_b200.data.loader import PackedRowLoader
    ld = PackedRowLoader(B, T, torch.device("cpu"), "train", seed=seed, rank=0)
    out = []
    for _ in range(n):
        r = ld.next().clone()
        out.append((r[:, :-1].contiguous(), r[:, 1:].long().contiguous()))
    return out


def _ours_tiny():
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.models.gpt import GPT
    cfg = preset("tiny")
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    return cfg, m


def test_state_dict_keys_match_reference():
    rtrain = import_reference()
    ref = build_reference_tiny(rtrain)
    _, ours = _ours_tiny()
    assert set(ref.state_dict().keys()) == set(ours.state_dict().keys())
    for k, v in ref.state_dict().items():
        assert ours.state_dict()[k].shape == v.shape, k


def test_init_rng_order_matches_reference():
    """Same seed -> bit-identical initial weights (construction + init_weights draw order)."""
    rtrain = import_reference()
    ref = build_reference_tiny(rtrain, seed=3)
    torch.manual_seed(3)
    _, ours = _ours_tiny()
    rs = ref.state_dict()
    for k, v in ours.state_dict().items():
        assert torch.equal(v, rs[k]), k


def test_forward_loss_matches_reference():
    rtrain = import_reference()
    ref = build_reference_tiny(rtrain)
    _, ours = _ours_tiny()
    ours.load_state_dict(ref.state_dict())
    x, y = _batches(1)[0]
    with torch.no_grad():
        lr_ = ref(x, y).item()
        lo = ours(x, y).item()
        logits_r = ref(x)
        logits_o = ours(x)
    assert abs(lr_ - lo) < 1e-5, (lr_, lo)
    assert (logits_r - logits_o).abs().max().item() < 1e-4


def _reference_step(rtrain, model, opt, x, y, step, n_steps):
    opt.zero_grad(set_to_none=True)
    loss = model(x, y)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(list(model.parameters()), rtrain.GRAD_CLIP, foreach=True)
    prog = step / n_steps
    for g in opt.param_groups:
        g["lr"] = g["initial_lr"]
        if g["kind"] == "muon":
            g["momentum"] = rtrain.muon_momentum(step, prog)
            g["weight_decay"] = rtrain.WEIGHT_DECAY * (1.0 - prog)
    opt.step()
    return loss.item()


def _ours_step(cfg, model, opt, x, y, step, n_steps):
    from trainium_frontier_b200.optim.schedules import muon_momentum
    opt.zero_grad_selective(True)
    loss = model(x, y)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(list(model.parameters()), cfg.grad_clip, foreach=True)
    prog = step / n_steps
    for g in opt.param_groups:
        g["lr"] = g["initial_lr"]
        if g["kind"] == "muon":
            g["momentum"] = muon_momentum(cfg, step, prog)
            g["weight_decay"] = cfg.weight_decay * (1.0 - prog)
    opt.step()
    return loss.item()


@pytest.mark.parametrize("n_steps", [20])
def test_training_loss_parity_ws1(n_steps):
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    rtrain = import_reference()
    ref = build_reference_tiny(rtrain)
    cfg, ours = _ours_tiny()
    ours.load_state_dict(ref.state_dict())
    opt_r = ref.setup_optimizer()
    opt_o = setup_optimizer(ours, cfg, compute_dtype=torch.float32)
    batches = _batches(n_steps)
    lr_hist, lo_hist = [], []
    for i, (x, y) in enumerate(batches):
        lr_hist.append(_reference_step(rtrain, ref, opt_r, x, y, i, n_steps))
        lo_hist.append(_ours_step(cfg, ours, opt_o, x, y, i, n_steps))
    for i, (a, b) in enumerate(zip(lr_hist, lo_hist)):
        assert math.isfinite(b)
        assert abs(a - b) <= 1e-3 * abs(a), (i, a, b)
    assert lo_hist[-1] < lo_hist[0] - 1.0
    # held-out bpb at equal training tokens, scored by the same trusted evaluation
    from trainium_frontier_b200.eval import evaluate_bpb
    with torch.no_grad():
        r_ref = evaluate_bpb(ref, None, 8, 256, "cpu", max_tokens=8192)
        r_our = evaluate_bpb(ours, None, 8, 256, "cpu", max_tokens=8192)
    assert r_ref["num_tokens"] == r_our["num_tokens"] >= 8192
    assert abs(r_ref["val_bpb"] - r_our["val_bpb"]) <= 1e-3 * r_ref["val_bpb"], (r_ref, r_our)
