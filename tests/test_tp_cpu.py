"""Tensor parallelism on CPU (gloo, world 2 = TP 2 x DP 1): the sharded block math and
the gradient scaling rule give the same loss and gradients as one process that runs the
whole micro-batch (the CUDA path fuses the same collectives into the GEMM kernels)."""
import os
import socket
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(**kw):
    from trainium_frontier_b200.config import preset
    return preset("tiny", grad_clip=0.0, clip_order="global", bucket_layers=2, **kw)


def _batch():
    g = torch.Generator().manual_seed(7)
    return torch.randint(1, 8192, (4, 257), generator=g)


def _worker(rank, world, port, out_dir, mode):
    import datetime
    sys.path.insert(0, ROOT)
    torch.set_num_threads(2)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from trainium_frontier_b200.engine import TrainEngine
    from trainium_frontier_b200.models.gpt import GPT
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    from trainium_frontier_b200.parallel.tensor_parallel import TPContext
    cfg = _cfg(tp=2, grad_sync=mode)
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    x = _batch()[2 * rank:2 * rank + 2]
    tpc = TPContext(2, torch.device("cpu"), 2 * 256, cfg.model_config().n_embd, 2 * cfg.model_config().n_layer)
    m.enable_tp(tpc)
    opt = setup_optimizer(m, cfg, torch.float32)
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 1, mode)
    losses = []
    grads = None
    for step in range(3):
        loss = eng.forward_backward([(x[:, :-1], x[:, 1:])])
        l = loss.detach().clone()
        dist.all_reduce(l)
        losses.append(float(l) / world)
        eng.sync_and_clip()
        if step == 0:
            grads = eng.layout.grad.clone()
        eng.optimizer_step()
    torch.save({"losses": losses, "grads": grads, "names": [n for n, _ in m.named_parameters()]},
               os.path.join(out_dir, f"tp_{rank}.pt"))
    dist.destroy_process_group()


def _single():
    from trainium_frontier_b200.engine import TrainEngine
    from trainium_frontier_b200.models.gpt import GPT
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    cfg = _cfg(grad_sync="none")
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    opt = setup_optimizer(m, cfg, torch.float32)
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 1, "none")
    x = _batch()
    losses, grads = [], None
    for step in range(3):
        losses.append(float(eng.forward_backward([(x[:, :-1], x[:, 1:])])))
        eng.sync_and_clip()
        if step == 0:
            grads = eng.layout.grad.clone()
        eng.optimizer_step()
    return losses, grads


def _run(tmp_path, mode):
    port = _port()
    mp.spawn(_worker, args=(2, port, str(tmp_path), mode), nprocs=2, join=True)
    return [torch.load(os.path.join(tmp_path, f"tp_{r}.pt")) for r in range(2)]


def test_tp2_matches_single_process(tmp_path):
    res = _run(tmp_path, "bucket")
    ref_losses, ref_grads = _single()
    for r in res:
        assert torch.equal(r["grads"], res[0]["grads"]), "TP replicas disagree"
    g = res[0]["grads"]
    rel = float((g - ref_grads).norm() / ref_grads.norm())
    assert rel < 1e-4, rel
    for a, b in zip(res[0]["losses"], ref_losses):
        assert abs(a - b) < 2e-4 * max(1.0, abs(b)), (res[0]["losses"], ref_losses)


def test_tp2_dist_muon_matches_single_process(tmp_path):
    res = _run(tmp_path, "dist_muon")
    ref_losses, _ = _single()
    for a, b in zip(res[0]["losses"], ref_losses):
        assert abs(a - b) < 2e-3 * max(1.0, abs(b)), (res[0]["losses"], ref_losses)
