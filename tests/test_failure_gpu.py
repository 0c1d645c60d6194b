"""Failure detection on the GPU without a fault: a bounded device wait that can never be
satisfied (a peer flag that nothing sets) must give up after its time budget, report an
error status the host reads, and leave the CUDA context usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_wait_runs_out_and_context_survives(cuda_device):
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops._ext import C, KernelTimeout, check_errors, err_word
    check_errors(cuda_device)
    mine = torch.zeros(8, dtype=torch.int32, device=cuda_device)      # this rank's signal pad
    ghost = torch.zeros(8, dtype=torch.int32, device=cuda_device)     # a "peer" that never runs
    err = err_word(cuda_device)
    t0 = time.time()
    C().symm_barrier([mine.data_ptr(), ghost.data_ptr()], 0, 1, err)
    with pytest.raises(KernelTimeout):
        check_errors(cuda_device)
    waited = time.time() - t0
    assert 1.0 < waited < 30.0, waited          # gave up after its ~2 s budget, did not hang
    assert int(mine[0]) == 1 and int(ghost[0]) == 1  # it did signal before waiting
    # the context is still usable: a tcgen05 GEMM gives the right answer afterwards
    a = torch.randn(256, 512, device=cuda_device).to(torch.bfloat16)
    w = torch.randn(384, 512, device=cuda_device).to(torch.bfloat16)
    y = gemm.linear_fwd(a, w)
    ref = a.float() @ w.float().t()
    assert float((y.float() - ref).norm() / ref.norm()) < 1e-2
    assert check_errors(cuda_device) == 0
