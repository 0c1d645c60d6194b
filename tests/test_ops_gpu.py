"""Numerics of the fused sm_100a ops against fp32 PyTorch references of the same ops."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / (b.abs().max() + 1e-8)).item()


def _grads(fn, *xs):
    xs = [x.detach().clone().requires_grad_(True) for x in xs]
    y = fn(*xs)
    return y, xs


def test_rmsnorm(cuda_device):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(0)
    for C in (256, 768, 1280, 1664):
        x = torch.randn(1000, C, device=cuda_device)
        g = torch.randn(1000, C, device=cuda_device)
        xb = x.to(BF).requires_grad_(True)
        y = ops.norm(xb)
        y.backward(g.to(BF))
        xr = x.to(BF).float().requires_grad_(True)
        yr = ref.norm(xr)
        yr.backward(g.to(BF).float())
        assert rel(y, yr) < 1e-2
        assert rel(xb.grad, xr.grad) < 2e-2


def test_mix_norm(cuda_device):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(1)
    M, C = 512, 1280
    x = torch.randn(M, C, device=cuda_device).to(BF)
    x0 = torch.randn(M, C, device=cuda_device).to(BF)
    lr = torch.tensor([0.9], device=cuda_device, requires_grad=True)
    l0 = torch.tensor([0.1], device=cuda_device, requires_grad=True)
    gx = torch.randn(M, C, device=cuda_device).to(BF)
    gh = torch.randn(M, C, device=cuda_device).to(BF)
    xa, x0a = x.clone().requires_grad_(True), x0.clone().requires_grad_(True)
    xm, h = ops.mix_norm(xa, x0a, lr, l0)
    (xm.float() * gx.float()).sum().add_((h.float() * gh.float()).sum()).backward()
    xr, x0r = x.float().requires_grad_(True), x0.float().requires_grad_(True)
    lrr = lr.detach().clone().requires_grad_(True)
    l0r = l0.detach().clone().requires_grad_(True)
    xmr, hr = ref.mix_norm(xr, x0r, lrr, l0r)
    (xmr * gx.float()).sum().add_((hr * gh.float()).sum()).backward()
    assert rel(xm, xmr) < 1e-2 and rel(h, hr) < 1e-2
    assert rel(xa.grad, xr.grad) < 2e-2
    assert rel(x0a.grad, x0r.grad) < 2e-2
    assert rel(lr.grad, lrr.grad) < 1e-2 and rel(l0.grad, l0r.grad) < 1e-2


def test_embed_norm(cuda_device):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(2)
    V, C, B, T = 8192, 1280, 4, 256
    wte = torch.randn(V, C, device=cuda_device, requires_grad=True)
    idx = torch.randint(0, V, (B, T + 1), device=cuda_device, dtype=torch.int32)[:, :-1]  # strided rows
    g = torch.randn(B, T, C, device=cuda_device).to(BF)
    y = ops.embed_norm(idx, wte, BF)
    y.backward(g)
    wr = wte.detach().clone().requires_grad_(True)
    yr = ref.norm(torch.nn.functional.embedding(idx.long(), wr).to(BF).float())
    yr.backward(g.float())
    assert rel(y, yr) < 1e-2
    assert rel(wte.grad, wr.grad) < 2e-2


def test_rope_norm(cuda_device):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(3)
    for D in (64, 128):
        B, T, H = 2, 256, 4
        t = torch.arange(T, dtype=torch.float32)
        inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        tab = torch.outer(t, inv)
        cos = tab.cos().to(BF)[None, :, None, :].to(cuda_device)
        sin = tab.sin().to(BF)[None, :, None, :].to(cuda_device)
        x = torch.randn(B, T, H, D, device=cuda_device).to(BF).requires_grad_(True)
        g = torch.randn(B, T, H, D, device=cuda_device).to(BF)
        y = ops.rope_norm(x, cos, sin)
        y.backward(g)
        xr = x.detach().float().requires_grad_(True)
        yr = ref.rope_norm(xr, cos.float(), sin.float())
        yr.backward(g.float())
        assert rel(y, yr) < 1e-2
        assert rel(x.grad, xr.grad) < 2e-2


@pytest.mark.parametrize("V", [8192, 1000])
def test_lm_head_softcap_ce(cuda_device, V):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(4)
    M, C = 1024, 768
    Vp = ((V + 63) // 64) * 64
    x = (torch.randn(M, C, device=cuda_device) * 2).to(BF).requires_grad_(True)
    w = (torch.randn(Vp, C, device=cuda_device) * 0.05).requires_grad_(True)
    tg = torch.randint(0, V, (4, M // 4), device=cuda_device)
    tg[0, :5] = -1
    loss = ops.lm_head_softcap_ce(x, w, tg, 15.0, V)
    (loss * 3.0).backward()
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().to(BF).float().requires_grad_(True)
    lr_ = ref.softcap_cross_entropy(ref.linear(xr, wr)[..., :V].float(), tg.view(-1), 15.0)
    (lr_ * 3.0).backward()
    assert abs(loss.item() - lr_.item()) < 2e-2 * max(1.0, abs(lr_.item()))
    assert rel(x.grad, xr.grad) < 3e-2
    assert rel(w.grad, wr.grad) < 3e-2


def test_mlp_relu2(cuda_device):
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(5)
    M, C = 1024, 768
    x = torch.randn(M, C, device=cuda_device).to(BF).requires_grad_(True)
    wf = (torch.randn(4 * C, C, device=cuda_device) * C ** -0.5).requires_grad_(True)
    wp = (torch.randn(C, 4 * C, device=cuda_device) * (4 * C) ** -0.5).requires_grad_(True)
    r = torch.randn(M, C, device=cuda_device).to(BF).requires_grad_(True)
    g = torch.randn(M, C, device=cuda_device).to(BF)
    y = ops.mlp_relu2(x, wf, wp, residual=r)
    y.backward(g)
    xr = x.detach().float().requires_grad_(True)
    wfr = wf.detach().to(BF).float().requires_grad_(True)
    wpr = wp.detach().to(BF).float().requires_grad_(True)
    rr = r.detach().float().requires_grad_(True)
    yr = ref.mlp_relu2(xr, wfr, wpr, residual=rr)
    yr.backward(g.float())
    assert rel(y, yr) < 2e-2
    assert rel(x.grad, xr.grad) < 3e-2
    assert rel(wf.grad, wfr.grad) < 3e-2
    assert rel(wp.grad, wpr.grad) < 3e-2
    assert rel(r.grad, rr.grad) < 1e-6


def test_attention_qkv(cuda_device):
    from trainium_frontier_b200 import ops
    torch.manual_seed(6)
    B, T, H, D = 2, 512, 4, 128
    t = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    tab = torch.outer(t, inv)
    cos = tab.cos().to(BF)[None, :, None, :].to(cuda_device)
    sin = tab.sin().to(BF)[None, :, None, :].to(cuda_device)
    qkv = torch.randn(B, T, 3 * H * D, device=cuda_device).to(BF).requires_grad_(True)
    g = torch.randn(B, T, H * D, device=cuda_device).to(BF)
    y = ops.attention_qkv(qkv, cos, sin, H, D, None)
    y.backward(g)
    qr = qkv.detach().float().cpu().requires_grad_(True)
    yr = ops.attention_qkv(qr, cos.float().cpu(), sin.float().cpu(), H, D, None)
    yr.backward(g.float().cpu())
    assert rel(y.cpu(), yr) < 2e-2
    assert rel(qkv.grad.cpu(), qr.grad) < 5e-2


def _rope_tables(T, D, device):
    t = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    tab = torch.outer(t, inv)
    return tab.cos().to(BF)[None, :, None, :].to(device), tab.sin().to(BF)[None, :, None, :].to(device)


def test_gemm_rope_epilogue(cuda_device):
    """QKV projection GEMM with RoPE + per-head RMSNorm in the epilogue vs fp32 torch."""
    from trainium_frontier_b200.ops import gemm
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(11)
    B, T, H, D, K = 2, 256, 3, 128, 320
    Cd = H * D
    cos, sin = _rope_tables(T, D, cuda_device)
    x = (torch.randn(B * T, K, device=cuda_device) * 0.5).to(BF)
    w = (torch.randn(3 * Cd, K, device=cuda_device) * K ** -0.5).to(BF)
    rstd = torch.empty(B * T * 2 * H, dtype=torch.float32, device=cuda_device)
    out = gemm.linear_rope_fwd(x, w, cos.reshape(T, D // 2).contiguous(), sin.reshape(T, D // 2).contiguous(),
                               T, 2 * Cd, rstd)
    torch.cuda.synchronize()
    raw = (x.float() @ w.float().t()).to(BF).float()           # what the epilogue rounds to first
    qk = raw[:, :2 * Cd].view(B, T, 2 * H, D)
    ref_qk = ref.rope_norm(qk, cos.float(), sin.float()).reshape(B * T, 2 * Cd)
    assert rel(out[:, :2 * Cd], ref_qk) < 1e-2
    assert rel(out[:, 2 * Cd:], raw[:, 2 * Cd:]) < 1e-2       # v columns untouched
    rot = ref.apply_rotary_emb(qk, cos.float(), sin.float())
    ref_r = torch.rsqrt(rot.pow(2).mean(-1) + torch.finfo(torch.float32).eps).reshape(-1)
    assert rel(rstd, ref_r) < 1e-3


def test_qkv_rope_attention_matches_unfused(cuda_device, monkeypatch):
    """The projection-fused RoPE + QK-norm attention path gives the same output and the
    same input / weight gradients as projection GEMM -> RoPE kernel -> attention."""
    from trainium_frontier_b200 import ops
    torch.manual_seed(12)
    B, T, H, D = 2, 256, 4, 128
    C = H * D
    cos, sin = _rope_tables(T, D, cuda_device)
    x = (torch.randn(B, T, C, device=cuda_device)).to(BF)
    ws = [(torch.randn(C, C, device=cuda_device) * C ** -0.5) for _ in range(3)]
    g = torch.randn(B, T, C, device=cuda_device).to(BF)

    def run(flag):
        monkeypatch.setenv("TFB_QKV_ROPE", flag)
        xa = x.clone().requires_grad_(True)
        wa = [w.clone().requires_grad_(True) for w in ws]
        y = ops.qkv_attention(xa, wa, cos, sin, H, D, None)
        y.backward(g)
        torch.cuda.synchronize()
        return y.detach(), xa.grad, [w.grad for w in wa]

    y1, dx1, dw1 = run("1")
    y0, dx0, dw0 = run("0")
    assert rel(y1, y0) < 2e-2
    assert rel(dx1, dx0) < 3e-2
    for a, b in zip(dw1, dw0):
        assert rel(a, b) < 3e-2


def test_adamw_multi(cuda_device):
    from trainium_frontier_b200.ops.optim_kernels import adamw_multi
    torch.manual_seed(7)
    shapes = [(300, 7), (1,), (8192, 33)]
    ps = [torch.randn(s, device=cuda_device) for s in shapes]
    gs = [torch.randn(s, device=cuda_device) for s in shapes]
    ms = [torch.randn(s, device=cuda_device).abs() * 0.1 for s in shapes]
    vs = [torch.randn(s, device=cuda_device).abs() * 0.1 for s in shapes]
    pr, mr, vr = [p.clone() for p in ps], [m.clone() for m in ms], [v.clone() for v in vs]
    lr = torch.tensor(0.01, device=cuda_device)
    b1, b2, eps, wd = 0.8, 0.95, 1e-10, 0.01
    bc1, bc2 = [1 - b1 ** 3] * 3, [1 - b2 ** 3] * 3
    adamw_multi(ps, gs, ms, vs, lr, b1, b2, eps, wd, bc1, bc2)
    torch._foreach_lerp_(mr, gs, 1 - b1)
    torch._foreach_lerp_(vr, torch._foreach_mul(gs, gs), 1 - b2)
    den = torch._foreach_div(vr, bc2)
    torch._foreach_sqrt_(den)
    torch._foreach_add_(den, eps)
    up = torch._foreach_div(mr, bc1)
    torch._foreach_div_(up, den)
    torch._foreach_mul_(pr, 1 - lr * wd)
    torch._foreach_mul_(up, lr)
    torch._foreach_sub_(pr, up)
    for a, b in zip(ps + ms + vs, pr + mr + vr):
        assert rel(a, b) < 1e-5


def test_newton_schulz(cuda_device):
    from trainium_frontier_b200.ops.newton_schulz import newton_schulz_gpu, newton_schulz_reference
    torch.manual_seed(8)
    for shape in [(6, 256, 256), (3, 1024, 256), (3, 256, 768)]:
        x = torch.randn(shape, device=cuda_device)
        x = x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)
        y = newton_schulz_gpu(x.to(BF), 5)
        yr = newton_schulz_reference(x.double(), 5)
        assert rel(y, yr) < 5e-2, shape
        # same spectrum as the fp64 reference iteration (Polar Express is not exactly orthogonal)
        s = torch.linalg.svdvals(y.float())
        sr = torch.linalg.svdvals(yr.float())
        assert (s - sr).abs().max().item() < 5e-2


def test_model_cpu_vs_gpu(cuda_device):
    """Same weights, same batch: bf16 GPU model vs fp32 CPU model (loss and grads)."""
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.models.gpt import GPT
    torch.manual_seed(9)
    cfg = preset("tiny", attn_cproj_init_scale=0.1)
    gc = cfg.model_config()
    cpu = GPT(gc, cfg)
    cpu.init_weights()
    # give the zero-init projections some weight so their gradients flow
    with torch.no_grad():
        for b in cpu.transformer.h:
            b.mlp.c_proj.weight.normal_(0, 0.02)
    gpu = GPT(gc, cfg)
    gpu.load_state_dict(cpu.state_dict())
    gpu.set_compute_dtype(BF)
    gpu.to(cuda_device)
    idx = torch.randint(1, 8192, (4, 257))
    x, y = idx[:, :-1], idx[:, 1:]
    lc = cpu(x, y)
    lc.backward()
    lg = gpu(x.to(cuda_device).to(torch.int32), y.to(cuda_device))
    lg.backward()
    assert abs(lc.item() - lg.item()) < 2e-2 * lc.item()
    pc = dict(cpu.named_parameters())
    errs, lam = {}, []
    for n, p in gpu.named_parameters():
        if pc[n].grad is None:
            continue
        assert p.grad is not None, n
        a, b = p.grad.cpu().float(), pc[n].grad.float()
        if n.endswith("_lambda"):
            lam.append((n, a.item(), b.item()))
            continue
        errs[n] = ((a - b).norm() / (b.norm() + 1e-12)).item()
    worst = sorted(errs.items(), key=lambda kv: -kv[1])[:5]
    assert worst[0][1] < 0.05, worst
    # The per-block scalars' gradients are dot products over the whole (bf16) residual
    # stream with heavy cancellation: compare on the scale of the largest of them.
    scale = max(abs(b) for _, _, b in lam)
    for n, a, b in lam:
        assert abs(a - b) < 0.15 * scale, (n, a, b, scale)


@pytest.mark.parametrize("K", [2, 4])
def test_causal_conv(cuda_device, K):
    """Depthwise causal conv1d kernel (forward, dx, deterministic dw) against the fp32
    conv1d of the same bf16-rounded inputs and weight."""
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(6)
    B, T, C = 3, 300, 1280
    x = torch.randn(B, T, C, device=cuda_device).to(BF)
    w = (torch.randn(C, 1, K, device=cuda_device) * 0.3).requires_grad_(True)
    g = torch.randn(B, T, C, device=cuda_device).to(BF)
    xb = x.clone().requires_grad_(True)
    y = ops.causal_conv(xb, w)
    y.backward(g)
    xr = x.float().requires_grad_(True)
    wr = w.detach().to(BF).float().requires_grad_(True)
    yr = ref.causal_conv(xr, wr)
    yr.backward(g.float())
    assert rel(y, yr) < 1e-2
    assert rel(xb.grad, xr.grad) < 1e-2
    assert rel(w.grad, wr.grad) < 1e-3
    dw1 = w.grad.clone()
    w.grad = None
    ops.causal_conv(x.clone().requires_grad_(True), w).backward(g)
    assert torch.equal(w.grad, dw1)  # the weight gradient is bitwise reproducible


@pytest.mark.parametrize("order", [2, 3])
def test_ngram_lookup(cuda_device, order):
    """Fused n-gram hash + gather against the reference hash and indexing; the backward's
    scatter-add against index_add into an fp32 table gradient."""
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(7)
    B, T, V, rows, Dn = 4, 512, 8192, 65521, 128
    idx = torch.randint(0, V, (B, T), device=cuda_device, dtype=torch.int32)
    table = torch.randn(rows, Dn, device=cuda_device).requires_grad_(True)
    primes = (31033, 53087, 71023)[:order]
    out = ops.ngram_lookup(idx, table, order, primes, rows, V, BF)
    rid = ref.ngram_rows(idx, order, primes, rows, V)
    assert torch.equal(out, table.detach()[rid].to(BF))
    g = torch.randn(B, T, Dn, device=cuda_device).to(BF)
    out.backward(g)
    gr = torch.zeros(rows, Dn, device=cuda_device).index_add_(0, rid.reshape(-1), g.reshape(-1, Dn).float())
    assert rel(table.grad, gr) < 1e-5


@pytest.mark.parametrize("shape", [(4, 256, 256), (3, 1024, 256), (2, 256, 768)])
def test_muon_owner_kernels_match_reference_math(cuda_device, shape):
    """The fused Muon owner path (momentum prologue, Frobenius normalisation, Newton-Schulz,
    NorMuon tail, apply) against the reference's op-by-op math on the same CUDA inputs."""
    from trainium_frontier_b200.optim.muon_adamw import _muon_math
    from trainium_frontier_b200.ops.optim_kernels import muon_owner_update
    torch.manual_seed(9)
    K, r, c = shape
    red_dim = -1 if r >= c else -2
    sshape = (K, r, 1) if red_dim == -1 else (K, 1, c)
    w = torch.randn(K, r, c, device=cuda_device) * 0.02
    g = torch.randn(K, r, c, device=cuda_device) * 0.01
    mb = torch.randn(K, r, c, device=cuda_device) * 0.01
    second = torch.rand(sshape, device=cuda_device) * 1e-3
    dev = lambda v: torch.tensor(v, dtype=torch.float32, device=cuda_device)  # noqa: E731
    lr, lrwd, mom, one_mom, one_b2 = dev(0.02), dev(0.02 * 0.2), dev(0.95), dev(0.05), dev(0.1)
    w1, mb1, s1 = w.clone(), mb.clone(), second.clone()
    _muon_math(w1, g.clone(), mb1, s1, mom, one_mom, lr, lrwd, 5, red_dim, one_b2, True, False)
    w2, mb2, s2 = w.clone(), mb.clone(), second.clone()
    muon_owner_update(g.clone(), mb2, s2, mom, one_mom, one_b2, 5, w=w2, lr=lr, lrwd=lrwd)
    torch.testing.assert_close(mb2, mb1, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(s2, s1, rtol=2e-2, atol=1e-6)
    # the applied step lr * u is ~1e-2 of w; compare the steps
    assert rel(w2 - w, w1 - w) < 3e-2
    # the bf16 update written to a buffer instead of applied
    out = torch.empty(K, r, c, device=cuda_device, dtype=BF)
    muon_owner_update(g.clone(), mb.clone(), second.clone(), mom, one_mom, one_b2, 5, out=out)
    upd = (w - w2)  # = bf16(lr) u + decay
    assert torch.isfinite(out.float()).all() and out.float().abs().max() > 0
    # bit-reproducible: replicas that each run the optimizer on identical gradients (the
    # bucketed all-reduce path) must keep identical fp32 masters
    out2 = torch.empty_like(out)
    muon_owner_update(g.clone(), mb.clone(), second.clone(), mom, one_mom, one_b2, 5, out=out2)
    assert torch.equal(out, out2)


def test_embed_grad_deterministic_with_frequent_tokens(cuda_device):
    """The sorted segmented embedding gradient: tokens repeated thousands of times (several
    chunks each, added in order) match the fp32 oracle, and two runs agree bit for bit."""
    from trainium_frontier_b200 import ops
    from trainium_frontier_b200.ops import reference as ref
    torch.manual_seed(11)
    V, C, B, T = 8192, 1280, 4, 2048
    # a skewed id stream: Zipf-like weights, id 1 about a third of all positions
    w = 1.0 / torch.arange(1, V + 1, dtype=torch.float64) ** 1.3
    idx = torch.multinomial(w, B * T, replacement=True).view(B, T).to(torch.int32).to(cuda_device)
    assert int((idx == 0).sum()) > 1000
    wte = torch.randn(V, C, device=cuda_device)
    g = torch.randn(B, T, C, device=cuda_device).to(BF)
    grads = []
    for _ in range(2):
        wt = wte.clone().requires_grad_(True)
        ops.embed_norm(idx, wt, BF).backward(g)
        grads.append(wt.grad)
    assert torch.equal(grads[0], grads[1])
    wr = wte.clone().requires_grad_(True)
    ref.norm(torch.nn.functional.embedding(idx.long(), wr).to(BF).float()).backward(g.float())
    assert rel(grads[0], wr.grad) < 2e-2
