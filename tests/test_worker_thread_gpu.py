"""The kernels work when their host code runs first on a thread that has done no CUDA work
yet: a fresh process whose first backward node is the fused relu² MLP (so the MLP
backward GEMM is the first CUDA work on PyTorch's autograd thread), and a fresh Python
thread whose first CUDA work is a GEMM.  Each runs in a child process, since the state
in question is per thread and per process; results are checked against fp32 PyTorch."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import sys, threading, torch
sys.path.insert(0, sys.argv[1])
from trainium_frontier_b200 import ops
from trainium_frontier_b200.ops import gemm
from trainium_frontier_b200.ops import reference as ref

def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).abs().max() / (b.abs().max() + 1e-8)).item()

dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
torch.manual_seed(0)
x = torch.randn(512, 256, device=dev).to(torch.bfloat16).requires_grad_(True)
w_fc = (torch.randn(1024, 256, device=dev) * 0.05).requires_grad_(True)
w_proj = (torch.randn(256, 1024, device=dev) * 0.05).requires_grad_(True)
y = ops.mlp_relu2(x, w_fc, w_proj)
g = torch.randn(y.shape, device=dev).to(torch.bfloat16)
torch.autograd.backward([y], [g])     # first backward node: the fused MLP
torch.cuda.synchronize()
xr = x.detach().float().cpu().requires_grad_(True)
yr = ref.mlp_relu2(xr, w_fc.detach().cpu(), w_proj.detach().cpu())
yr.backward(g.float().cpu())
e_y, e_dx = rel(y, yr), rel(x.grad, xr.grad)

a = torch.randn(384, 512, device=dev).to(torch.bfloat16)
b = torch.randn(256, 512, device=dev).to(torch.bfloat16)
out = {}
def work():
    out["y"] = gemm.linear_fwd(a, b)   # first CUDA work of this thread
    torch.cuda.synchronize()
t = threading.Thread(target=work)
t.start()
t.join()
e_t = rel(out["y"], a.float() @ b.float().t())
print("ERRS", e_y, e_dx, e_t, flush=True)
assert e_y < 2e-2 and e_dx < 3e-2 and e_t < 1e-2, (e_y, e_dx, e_t)
print("CHILD_OK", flush=True)
'''


def test_first_cuda_work_on_a_fresh_thread(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    env = dict(os.environ, PYTHONFAULTHANDLER="1")
    p = subprocess.run(["timeout", "-k", "10", "240", sys.executable, str(script), ROOT], env=env,
                       capture_output=True, text=True)
    assert p.returncode == 0 and "CHILD_OK" in p.stdout, p.stdout[-2000:] + "\n" + p.stderr[-4000:]
