"""Engine layout (flat buffers, buckets, fused views) and equivalence to the plain loop."""
import torch

from trainium_frontier_b200.config import preset
from trainium_frontier_b200.engine import TrainEngine
from trainium_frontier_b200.models.gpt import GPT
from trainium_frontier_b200.optim.muon_adamw import setup_optimizer


def _model(seed=0, **kw):
    cfg = preset("tiny", **kw)
    torch.manual_seed(seed)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    return cfg, m


def test_layout_views_and_buckets():
    cfg, m = _model(bucket_layers=2)
    opt = setup_optimizer(m, cfg, torch.float32)
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 1)
    lay = eng.layout
    for p in m.parameters():
        assert p.data.data_ptr() >= lay.data.data_ptr()
        assert p.grad is not None and p.grad.data_ptr() >= lay.grad.data_ptr()
    assert len(lay.buckets) == 3  # two 2-layer chunks + the rest
    # every Muon group splits into contiguous runs per chunk
    for g in opt.param_groups:
        if g["kind"] == "muon":
            runs = opt._runs(g["params"])
            assert len(runs) == 2


def test_engine_matches_plain_loop():
    cfg, m1 = _model(seed=1)
    _, m2 = _model(seed=1)
    x = torch.randint(1, 8192, (8, 257))
    opt1 = setup_optimizer(m1, cfg, torch.float32)
    opt2 = setup_optimizer(m2, cfg, torch.float32)
    eng = TrainEngine(m2, opt2, cfg, torch.device("cpu"), 1)
    for step in range(3):
        opt1.zero_grad_selective(True)
        l1 = m1(x[:, :-1], x[:, 1:])
        l1.backward()
        torch.nn.utils.clip_grad_norm_(list(m1.parameters()), cfg.grad_clip)
        opt1.step()
        l2 = eng.forward_backward([(x[:, :-1], x[:, 1:])])
        eng.sync_and_clip()
        eng.optimizer_step()
        assert abs(l1.item() - l2.item()) < 1e-4 * abs(l1.item()), (step, l1.item(), l2.item())
    for (n, a), b in zip(m1.named_parameters(), m2.parameters()):
        assert torch.allclose(a, b, rtol=1e-2, atol=5e-4), n


def test_train_main_smoke(tmp_path, monkeypatch):
    from trainium_frontier_b200 import train
    out = tmp_path / "out"
    train.main(["--depth", "2", "--n-embd", "128", "--head-dim", "64", "--seq-len", "128",
                "--device-batch-size", "2", "--pack-factor", "1", "--total-batch-size", "256",
                "--num-steps", "3", "--progress-mode", "steps", "--out-dir", str(out),
                "--eval-tokens", "512", "--rope-base", "10000"])
    assert (out / "final.pt").exists()


def test_adamw_every_n_accumulates_between_updates():
    """With AdamW updating every 2nd step, embedding / lm_head stay frozen on the odd steps
    while their gradients accumulate; Muon matrices move every step."""
    import torch
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.train import Trainer
    cfg = preset("tiny", depth=2, progress_mode="steps", num_steps=8, device_batch_size=2,
                 total_batch_size=2 * 256 * 2, grad_sync="none", adam_every_n=2, grad_clip=0.0)
    tr = Trainer(cfg, torch.device("cpu"))
    wte = tr.model.transformer.wte.weight
    cq = tr.model.transformer.h[0].attn.c_q.weight
    w0, q0 = wte.detach().clone(), cq.detach().clone()
    tr.train_step()
    g1 = wte.grad.detach().clone()
    assert torch.equal(wte.detach(), w0), "AdamW params must not move on a non-update step"
    assert not torch.equal(cq.detach(), q0), "Muon params move every step"
    tr.train_step()
    assert not torch.equal(wte.detach(), w0), "AdamW applies on the second step"
    # the applied gradient was the sum of both steps' gradients
    assert float((wte.grad - g1).abs().sum()) > 0 and float(g1.abs().sum()) > 0
