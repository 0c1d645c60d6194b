"""tcgen05 flash attention (forward + backward) against an fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, causal, scale):
    # q, k, v [B, T, H, D] fp32
    s = torch.einsum("bthd,bshd->bhts", q, k) * scale
    if causal:
        T = q.shape[1]
        mask = torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    p = s.softmax(-1)
    o = torch.einsum("bhts,bshd->bthd", p, v)
    lse = torch.logsumexp(s, -1)  # [B, H, T]
    return o, lse


@pytest.mark.parametrize("B,T,H,D,causal,kgrow", [(2, 256, 2, 128, True, 0.0), (1, 512, 3, 64, True, 0.0),
                                                  (2, 384, 2, 128, False, 0.0), (1, 1024, 2, 128, True, 0.0),
                                                  (2, 512, 2, 128, False, 0.0), (1, 2048, 1, 128, True, 0.0),
                                                  (1, 1024, 2, 128, True, 3.0)])
def test_flash_fwd_bwd(cuda_device, B, T, H, D, causal, kgrow):
    """T % 256 == 0 with D = 128 runs the two-query-tile forward; kgrow > 0 scales the keys
    up along the sequence so the running row max keeps growing (exercises the O rescale)."""
    from trainium_frontier_b200.ops._ext import check_errors
    from trainium_frontier_b200.ops.flash_attention import flash_bwd, flash_fwd
    torch.manual_seed(0)
    scale = D ** -0.5
    q = torch.randn(B, T, H, D, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(B, T, H, D, device=cuda_device)
    if kgrow:
        k = k * (1.0 + kgrow * torch.arange(T, device=cuda_device) / T).view(1, T, 1, 1)
    k = k.to(torch.bfloat16)
    v = torch.randn(B, T, H, D, device=cuda_device).to(torch.bfloat16)
    do = torch.randn(B, T, H, D, device=cuda_device).to(torch.bfloat16)
    M = B * T
    o, lse = flash_fwd(q.view(M, H * D), k.view(M, H * D), v.view(M, H * D), B, T, H, D, scale, causal)
    check_errors()
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref, lse_ref = _ref(qf, kf, vf, causal, scale)
    err_o = (o.view(B, T, H, D).float() - o_ref).abs().max().item()
    assert err_o < 2e-2, err_o
    err_l = (lse.view(B, H, T) - lse_ref).abs().max().item()
    assert err_l < 1e-2, err_l
    o_ref.backward(do.float())
    dq, dk, dv = flash_bwd(q.view(M, H * D), k.view(M, H * D), v.view(M, H * D), o, do.view(M, H * D), lse,
                           B, T, H, D, scale, causal)
    check_errors()
    for name, a, b in (("dq", dq, qf.grad), ("dk", dk, kf.grad), ("dv", dv, vf.grad)):
        a = a.view(B, T, H, D).float()
        rel = ((a - b).norm() / b.norm()).item()
        assert rel < 2e-2, (name, rel)


def test_flash_strided_qkv_views(cuda_device):
    """q / k / v as column slices of one [M, 3C] buffer (the fused projection layout)."""
    from trainium_frontier_b200.ops.flash_attention import flash_fwd
    torch.manual_seed(1)
    B, T, H, D = 2, 256, 3, 128
    Cd = H * D
    buf = torch.randn(B * T, 3 * Cd, device=cuda_device).to(torch.bfloat16)
    o, _ = flash_fwd(buf[:, :Cd], buf[:, Cd:2 * Cd], buf[:, 2 * Cd:], B, T, H, D, D ** -0.5, True)
    q, k, v = (buf[:, i * Cd:(i + 1) * Cd].float().view(B, T, H, D) for i in range(3))
    o_ref, _ = _ref(q, k, v, True, D ** -0.5)
    assert (o.view(B, T, H, D).float() - o_ref).abs().max().item() < 2e-2
