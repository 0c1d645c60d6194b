"""Decode GEMM (swapped-operand tcgen05 tiles, cluster split-K reduced in distributed
shared memory, fused epilogues) against fp32 PyTorch references of the same ops."""
import pytest
import torch

pytestmark = pytest.mark.gpu

PLAIN, RES, RELU2, MIX, QKV = 0, 1, 2, 3, 4
EPS = torch.finfo(torch.float32).eps


def _rows(x):
    return torch.rsqrt(x.float().square().mean(-1, keepdim=True) + EPS)


def _call(x, w, out, epi, row_norm=False, R=None, X0=None, lr=None, l0=None, tau=0.0, cos=None, sin=None, pos=None,
          kc=None, vc=None, H=0, split=0, pdl=False):
    from trainium_frontier_b200.ops._ext import C, err_word
    C().decode_gemm(x, w, out, epi, row_norm, R, X0, lr, l0, tau, cos, sin, pos, kc, vc, H, split, pdl,
                    err_word(x.device))


def _close(got, ref, tol=2e-2):
    err = (got.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("M,N,K", [(1, 1280, 1280), (7, 384, 320), (32, 3840, 1280), (33, 1280, 5120),
                                   (64, 5120, 1280), (100, 640, 640), (128, 1280, 2560)])
@pytest.mark.parametrize("row_norm", [False, True])
def test_decode_gemm_plain(cuda_device, M, N, K, row_norm):
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = (torch.randn(N, K, device=cuda_device) * K ** -0.5).bfloat16()
    ref = x.float() @ w.float().t()
    if row_norm:
        ref = ref * _rows(x)
    for split in (0, 1, 2, 8):
        if split and split > (K + 63) // 64:
            continue
        for pdl in (False, True):
            out = torch.full((M, N), float("nan"), device=cuda_device).bfloat16()
            _call(x, w, out, PLAIN, row_norm, split=split, pdl=pdl)
            check_errors()
            _close(out, ref)


@pytest.mark.parametrize("M", [3, 32])
def test_decode_gemm_epilogues(cuda_device, M):
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(M)
    N, K = 1280, 5120
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = (torch.randn(N, K, device=cuda_device) * K ** -0.5).bfloat16()
    r = torch.randn(M, N, device=cuda_device).bfloat16()
    x0 = torch.randn(M, N, device=cuda_device).bfloat16()
    lr = torch.tensor([0.9], device=cuda_device)
    l0 = torch.tensor([0.3], device=cuda_device)
    acc = x.float() @ w.float().t()
    out = torch.empty(M, N, device=cuda_device).bfloat16()
    _call(x, w, out, RES, R=r, pdl=True)
    _close(out, acc + r.float())
    for tau in (0.0, 0.25):
        _call(x, w, out, RELU2, True, tau=tau)
        h = (acc * _rows(x)).bfloat16().float() - tau
        _close(out, torch.relu(h).square())
    _call(x, w, out, MIX, R=r, X0=x0, lr=lr, l0=l0)
    ref = 0.9 * (acc + r.float()).bfloat16().float() + 0.3 * x0.float()
    _close(out, ref)
    check_errors()


@pytest.mark.parametrize("layout", ["token", "head"])
def test_decode_gemm_qkv_rope_cache(cuda_device, layout):
    """QKV epilogue: row norm, RoPE at the device-side position, QK-norm, q to `out`,
    k and v rows into the caches at that position (nothing else of the caches moves);
    token-major [B, T, H*D] and head-major [B, H, T, D] caches."""
    from trainium_frontier_b200.ops import reference as ref_ops
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(11)
    M, H, D, K, Tmax, P = 5, 2, 128, 256, 24, 9
    N = 3 * H * D
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = (torch.randn(N, K, device=cuda_device) * K ** -0.5).bfloat16()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=cuda_device).float() / D))
    ang = torch.outer(torch.arange(Tmax, device=cuda_device).float(), inv)
    cos, sin = ang.cos().bfloat16().contiguous(), ang.sin().bfloat16().contiguous()
    kc = torch.randn(M + 1, Tmax, H * D, device=cuda_device).bfloat16()
    vc = torch.randn(M + 1, Tmax, H * D, device=cuda_device).bfloat16()
    kc0, vc0 = kc.clone(), vc.clone()
    pos = torch.tensor([P], dtype=torch.int32, device=cuda_device)
    q = torch.empty(M, H * D, device=cuda_device).bfloat16()
    if layout == "head":
        kh = kc.view(M + 1, Tmax, H, D).transpose(1, 2).contiguous()
        vh = vc.view(M + 1, Tmax, H, D).transpose(1, 2).contiguous()
        _call(x, w, q, QKV, True, cos=cos, sin=sin, pos=pos, kc=kh, vc=vh, H=H, pdl=True)
        kc.copy_(kh.transpose(1, 2).reshape(M + 1, Tmax, H * D))
        vc.copy_(vh.transpose(1, 2).reshape(M + 1, Tmax, H * D))
    else:
        _call(x, w, q, QKV, True, cos=cos, sin=sin, pos=pos, kc=kc, vc=vc, H=H, pdl=True)
    check_errors()
    qkv = ((x.float() @ w.float().t()) * _rows(x)).bfloat16().float()
    qr, kr, vr = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]

    def rn(t):
        t = t.view(M, H, D)
        return ref_ops.rope_norm(t, cos[P].float(), sin[P].float()).reshape(M, H * D)
    _close(q, rn(qr))
    _close(kc[:M, P], rn(kr))
    _close(vc[:M, P], vr)
    # every other cache row is untouched
    mask = torch.ones(M + 1, Tmax, dtype=torch.bool, device=cuda_device)
    mask[:M, P] = False
    assert torch.equal(kc[mask], kc0[mask]) and torch.equal(vc[mask], vc0[mask])


def test_decode_gemm_graph_replay(cuda_device):
    """Captured once, replayed many times: nothing is allocated or re-zeroed per call."""
    from trainium_frontier_b200.ops._ext import check_errors
    torch.manual_seed(3)
    M, N, K = 32, 3840, 1280
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = (torch.randn(N, K, device=cuda_device) * K ** -0.5).bfloat16()
    r = torch.randn(M, N, device=cuda_device).bfloat16()
    out = torch.empty(M, N, device=cuda_device).bfloat16()
    _call(x, w, out, RES, R=r, pdl=True)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _call(x, w, out, RES, R=r, pdl=True)
    for _ in range(5):
        x.normal_()
        g.replay()
        torch.cuda.synchronize()
        _close(out, x.float() @ w.float().t() + r.float())
    check_errors()
    del g
