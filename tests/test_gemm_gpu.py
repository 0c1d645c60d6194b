"""tcgen05 GEMM numerics against an fp32 PyTorch reference of the same product."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().t()


def _check(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1000, 1280, 1280),
                                   (4096, 3840, 1280), (333, 200, 72), (64, 128, 8192)])
def test_linear_fwd(cuda_device, M, N, K):
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(0)
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    y = gemm.linear_fwd(x, w)
    check_errors()
    _check(y, _ref(x, w))
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    y2 = gemm.linear_fwd(x, w, residual=r)
    _check(y2, _ref(x, w) + r.float())


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (2048, 5120, 1280), (200, 1000, 96)])
def test_relu2_fwd_bwd(cuda_device, M, N, K):
    from trainium_frontier_b200.ops import gemm
    torch.manual_seed(1)
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    act, h = gemm.linear_relu2_fwd(x, w)
    href = _ref(x, w)
    _check(h, href)
    _check(act, torch.relu(href) ** 2)
    dy = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    # dh = (dy @ w) * 2 relu(h) with w viewed [N, K] -> here dact[M,N] = dy2[M,K'] @ W2[K',N]
    w2 = torch.randn(K, N, device=cuda_device, dtype=torch.bfloat16) * N ** -0.5
    dact_ref = dy.float() @ w2.float()
    dh = gemm.linear_dx(dy, w2, relu2_h=h)
    _check(dh, dact_ref * 2 * torch.relu(h.float()))


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (4096, 1280, 1280), (8192, 1280, 5120), (300, 136, 72)])
def test_linear_dx_dw(cuda_device, M, N, K):
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(2)
    dy = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * N ** -0.5
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    dx = gemm.linear_dx(dy, w)
    _check(dx, dy.float() @ w.float())
    g = torch.zeros(N, K, device=cuda_device, dtype=torch.float32)
    gemm.linear_dw(dy, x, g, accumulate=True)
    ref = dy.float().t() @ x.float()
    _check(g, ref)
    gemm.linear_dw(dy, x, g, accumulate=True)
    _check(g, 2 * ref)
    gemm.linear_dw(dy, x, g, accumulate=False, split_k=1)
    _check(g, ref)
    check_errors()


@pytest.mark.parametrize("M,N,K", [(32, 3840, 1280), (8, 1280, 5120), (17, 8192, 1280), (32, 200, 136)])
def test_linear_decode_split_k(cuda_device, M, N, K):
    """Few-row GEMM in one launch: split-K partial sums finished (plain / + residual / relu^2)
    by the last split, the workspace left zeroed for the next call."""
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(3)
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    r = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    cache = {}
    ref = _ref(x, w)
    for _ in range(2):  # the second round checks that the first left ws / counters clean
        _check(gemm.linear_decode(x, w, cache), ref)
        _check(gemm.linear_decode(x, w, cache, residual=r), ref + r.float())
        _check(gemm.linear_decode(x, w, cache, relu2=True), torch.relu(ref.bfloat16().float()) ** 2)
    check_errors()
    ws, cnt, _split = next(iter(cache.values()))
    assert float(ws.abs().sum()) == 0.0 and int(cnt.abs().sum()) == 0


@pytest.mark.parametrize("M", [130, 384, 640])
def test_pair_tiles_row_tails(cuda_device, M):
    """256-wide tiles run on CTA pairs (tcgen05 cta_group::2, 256 rows per pair): row counts
    that leave the second CTA of the last pair partly or wholly past M."""
    from trainium_frontier_b200.ops import gemm
    torch.manual_seed(4)
    N, K = 512, 320
    x = torch.randn(M, K, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    _check(gemm.linear_fwd(x, w), _ref(x, w))
    dy = torch.randn(M, N, device=cuda_device, dtype=torch.bfloat16)
    _check(gemm.linear_dx(dy, w), dy.float() @ w.float())
    g = torch.zeros(N, K, device=cuda_device, dtype=torch.float32)
    gemm.linear_dw(dy, x, g, accumulate=False, split_k=1)
    _check(g, dy.float().t() @ x.float())


def test_pair_tiles_batched(cuda_device):
    """Batched products of the Newton-Schulz iteration (all three operand layouts) on CTA
    pairs, with a batch whose row count is not a multiple of 256."""
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(5)
    Bt, M, N, K = 3, 640, 512, 384
    a = torch.randn(Bt, M, K, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(Bt, N, K, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    r = torch.randn(Bt, M, N, device=cuda_device, dtype=torch.bfloat16)
    out = torch.empty(Bt, M, N, device=cuda_device, dtype=torch.bfloat16)
    gemm.bmm_nt(a, b, out, residual=r, alpha=0.5, rcoef=2.0)
    _check(out, 0.5 * (a.float() @ b.float().mT) + 2.0 * r.float())
    bk = torch.randn(Bt, K, N, device=cuda_device, dtype=torch.bfloat16) * K ** -0.5
    gemm.bmm_nn(a, bk, out)
    _check(out, a.float() @ bk.float())
    at = torch.randn(Bt, K, M, device=cuda_device, dtype=torch.bfloat16)
    gemm.bmm_tn(at, bk, out)
    _check(out, at.float().mT @ bk.float())
    check_errors()
