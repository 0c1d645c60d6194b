"""Pipeline parallelism on CPU (gloo, 2 stages): GPipe over isend / irecv gives the same
losses and gradients as one process running the whole model on the same micro-batches."""
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
    return preset("tiny", depth=3, grad_clip=0.0, clip_order="global", bucket_layers=2, **kw)


def _batches():
    g = torch.Generator().manual_seed(11)
    x = torch.randint(1, 8192, (3, 2, 257), generator=g)   # 3 micro-batches of 2 rows
    return [(r[:, :-1], r[:, 1:]) for r in x]


def _worker(rank, world, port, out_dir):
    import datetime
    sys.path.insert(0, ROOT)
    torch.set_num_threads(2)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from trainium_frontier_b200.engine import TrainEngine
    from trainium_frontier_b200.models.gpt import GPT
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    from trainium_frontier_b200.parallel.pipeline import PipelineContext
    cfg = _cfg(pp=2, grad_sync="bucket")
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    m.enable_pp(PipelineContext(2, cfg.model_config().n_layer))
    opt = setup_optimizer(m, cfg, torch.float32)
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 3, "bucket")
    losses, grads = [], None
    for step in range(3):
        losses.append(float(eng.forward_backward(_batches())))
        eng.sync_and_clip()
        if step == 0:
            grads = eng.layout.grad.clone()
        eng.optimizer_step()
    torch.save({"losses": losses, "grads": grads}, os.path.join(out_dir, f"pp_{rank}.pt"))
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
    eng = TrainEngine(m, opt, cfg, torch.device("cpu"), 3, "none")
    losses, grads = [], None
    for step in range(3):
        losses.append(float(eng.forward_backward(_batches())))
        eng.sync_and_clip()
        if step == 0:
            grads = eng.layout.grad.clone()
        eng.optimizer_step()
    return losses, grads


def test_pp2_matches_single_process(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    res = [torch.load(os.path.join(tmp_path, f"pp_{r}.pt")) for r in range(2)]
    ref_losses, ref_grads = _single()
    assert torch.equal(res[0]["grads"], res[1]["grads"]), "pipeline ranks disagree after the sync"
    rel = float((res[0]["grads"] - ref_grads).norm() / ref_grads.norm())
    assert rel < 1e-4, rel
    for r in res:
        for a, b in zip(r["losses"], ref_losses):
            assert abs(a - b) < 2e-4 * max(1.0, abs(b)), (r["losses"], ref_losses)
