"""Pipeline parallelism on 2 GPUs (NCCL p2p): a 2-stage GPipe step follows single-GPU
training of the same micro-batches.  Skipped with fewer than two GPUs."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r'''
import faulthandler, json, os, sys, torch, torch.distributed as dist
faulthandler.enable()   # a host-side crash in a rank prints its Python stack
sys.path.insert(0, os.environ["TFB_ROOT"])
from trainium_frontier_b200.config import preset
from trainium_frontier_b200.runtime import init_runtime
from trainium_frontier_b200.engine import TrainEngine
from trainium_frontier_b200.models.gpt import GPT
from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
from trainium_frontier_b200.parallel.pipeline import PipelineContext
from trainium_frontier_b200.ops._ext import check_errors
ddp, rank, local, world, dev = init_runtime("cuda", 0, timeout_s=120)
cfg = preset("tiny", depth=4, n_embd=256, head_dim=128, seq_len=256, grad_clip=1.0, clip_order="global",
             bucket_layers=2, pp=2, grad_sync="bucket")
torch.manual_seed(0)
m = GPT(cfg.model_config(), cfg).to(dev)
m.set_compute_dtype(torch.bfloat16)
m.init_weights()
m.enable_pp(PipelineContext(2, 4))
opt = setup_optimizer(m, cfg, compute_dtype=torch.bfloat16)
eng = TrainEngine(m, opt, cfg, dev, 2, "bucket")
gen = torch.Generator().manual_seed(7)
xb = torch.randint(1, 8192, (2, 2, 257), generator=gen).to(dev)
batches = [(r[:, :-1], r[:, 1:]) for r in xb]
losses = []
for step in range(4):
    print("STEP", step, flush=True)
    losses.append(float(eng.forward_backward(batches)))
    eng.sync_and_clip()
    eng.optimizer_step()
flat = eng.layout.data
chk = torch.stack([flat.double().sum(), flat.double().square().sum()])
allc = [torch.zeros_like(chk) for _ in range(world)]
dist.all_gather(allc, chk)
check_errors(dev)
if rank == 0:
    print("RESULT " + json.dumps({"losses": losses, "checks": [c.tolist() for c in allc]}))
dist.destroy_process_group()
'''


def test_pp2_matches_single_gpu(tmp_path):
    sys.path.insert(0, ROOT)
    script = tmp_path / "pp_worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, TFB_ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29547", str(script)]
    p = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-2000:] + "\n" + p.stderr[-6000:]
    res = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["checks"][0] == res["checks"][1]
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.engine import TrainEngine
    from trainium_frontier_b200.models.gpt import GPT
    from trainium_frontier_b200.optim.muon_adamw import setup_optimizer
    dev = torch.device("cuda", 0)
    cfg = preset("tiny", depth=4, n_embd=256, head_dim=128, seq_len=256, grad_clip=1.0, clip_order="global",
                 bucket_layers=2, grad_sync="none")
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg).to(dev)
    m.set_compute_dtype(torch.bfloat16)
    m.init_weights()
    opt = setup_optimizer(m, cfg, compute_dtype=torch.bfloat16)
    eng = TrainEngine(m, opt, cfg, dev, 2, "none")
    gen = torch.Generator().manual_seed(7)
    xb = torch.randint(1, 8192, (2, 2, 257), generator=gen).to(dev)
    batches = [(r[:, :-1], r[:, 1:]) for r in xb]
    ref = []
    for _ in range(4):
        ref.append(float(eng.forward_backward(batches)))
        eng.sync_and_clip()
        eng.optimizer_step()
    for a, b in zip(res["losses"][:3], ref[:3]):
        assert abs(a - b) < 2e-2 * abs(b), (res["losses"], ref)
