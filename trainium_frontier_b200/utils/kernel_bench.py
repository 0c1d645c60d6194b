"""Kernel micro-benchmarks: CUDA-event timing of the hot kernels against the roofline.

Usage: ``python -m trainium_frontier_b200.utils.kernel_bench [gemm|attn|decode|all] [--json PATH]``

Each case: 3+ warm-up launches, then timed launches with an L2 flush (a write of a
buffer larger than the 126 MB L2) between them, CUDA events on the launching stream
with a synchronize on both sides.  Reports achieved TFLOP/s or GB/s and the fraction
of the measured peaks in MEASURED_PEAKS.json (the torch cuBLAS GEMM is timed the same
way alongside as a reference point).

Reference counterparts: its research micro-benchmarks (``research/scratch/muon_nki_bench.py``,
``research/scratch/embed_gather_bench.py``) time the Muon and embedding-gather kernels,
which this file does not cover; here the Newton-Schulz GEMMs and the embedding kernels
are timed inside their step phases by ``utils/profile_step.py`` (and listed per launch
by an ``ncu`` launch capture of it).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Timer:
    def __init__(self, device):
        self.device = device
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def time(self, fn, iters: int = 10, warmup: int = 3, flush: bool = True) -> float:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(self.device)
        total = 0.0
        for _ in range(iters):
            if flush:
                self.flush.fill_(1.0)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize(self.device)
            total += s.elapsed_time(e)
        return total / iters


def bench_gemm(dev, peaks, shapes=None):
    from ..ops import gemm
    t = Timer(dev)
    rows = []
    shapes = shapes or [
        ("d20 qkv fwd", "fwd", 65536, 3840, 1280),
        ("d20 proj fwd", "fwd", 65536, 1280, 1280),
        ("d20 fc fwd relu2", "relu2", 65536, 5120, 1280),
        ("d20 mlp proj fwd", "fwd", 65536, 1280, 5120),
        ("d20 lm_head fwd", "fwd", 65536, 8192, 1280),
        ("d20 fc dx", "dx", 65536, 5120, 1280),
        ("d20 fc dW", "dw", 65536, 5120, 1280),
        ("d20 qkv dW", "dw", 65536, 3840, 1280),
        ("square 8192", "fwd", 8192, 8192, 8192),
    ]
    for name, kind, M, N, K in shapes:
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        w = torch.randn(N, K, device=dev, dtype=torch.bfloat16)
        dy = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        g = torch.zeros(N, K, device=dev, dtype=torch.float32)
        if kind == "fwd":
            ours = lambda: gemm.linear_fwd(x, w)
            ref = lambda: torch.matmul(x, w.t())
        elif kind == "relu2":
            ours = lambda: gemm.linear_relu2_fwd(x, w)
            ref = lambda: torch.relu(torch.matmul(x, w.t())).square()
        elif kind == "dx":
            ours = lambda: gemm.linear_dx(dy, w)
            ref = lambda: torch.matmul(dy, w)
        else:
            ours = lambda: gemm.linear_dw(dy, x, g)
            ref = lambda: g.add_(torch.matmul(dy.t(), x).float())
        flops = 2.0 * M * N * K
        t_ours = t.time(ours)
        t_ref = t.time(ref)
        rows.append(dict(name=name, M=M, N=N, K=K, ms=t_ours, tflops=flops / t_ours / 1e9,
                         frac_of_measured=flops / t_ours / 1e9 / peaks["bf16_tflops"],
                         torch_ms=t_ref, torch_tflops=flops / t_ref / 1e9))
        del x, w, dy, g
    return rows


def bench_attention(dev, peaks, B=16, T=2048, H=10, D=128):
    """Causal flash attention fwd / bwd at the d20 shape (FLOPs counted causally)."""
    from ..ops.flash_attention import flash_bwd, flash_fwd
    t = Timer(dev)
    M = B * T
    q, k, v, do = (torch.randn(M, H * D, device=dev, dtype=torch.bfloat16) for _ in range(4))
    o, lse = flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)
    fl_fwd = 4.0 * B * H * T * T * D / 2
    t_f = t.time(lambda: flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True))
    t_b = t.time(lambda: flash_bwd(q, k, v, o, do, lse, B, T, H, D, D ** -0.5, True))
    qs, ks, vs = (x.view(B, T, H, D).transpose(1, 2).detach().requires_grad_(True) for x in (q, k, v))
    dos = do.view(B, T, H, D).transpose(1, 2)
    sdpa = torch.nn.functional.scaled_dot_product_attention
    with torch.no_grad():
        t_ref = t.time(lambda: sdpa(qs, ks, vs, is_causal=True))
    # the library's backward alone: forward once, then time autograd.grad over the saved graph
    o_ref = sdpa(qs, ks, vs, is_causal=True)
    t_ref_b = t.time(lambda: torch.autograd.grad(o_ref, (qs, ks, vs), dos, retain_graph=True))
    rows = [dict(name="flash fwd", ms=t_f, tflops=fl_fwd / t_f / 1e9, torch_sdpa_ms=t_ref,
                 torch_sdpa_tflops=fl_fwd / t_ref / 1e9),
            dict(name="flash bwd", ms=t_b, tflops=2.5 * fl_fwd / t_b / 1e9, torch_sdpa_ms=t_ref_b,
                 torch_sdpa_tflops=2.5 * fl_fwd / t_ref_b / 1e9)]
    for r in rows:
        r["frac_of_measured"] = r["tflops"] / peaks["bf16_tflops"]
    return rows


def one_kernel(case: str, dev):
    """A single small launch after three warm-ups (for ncu captures of one kernel)."""
    from ..ops import gemm
    from ..ops.flash_attention import flash_bwd, flash_fwd
    if case == "gemm":
        x = torch.randn(16384, 1280, device=dev, dtype=torch.bfloat16)
        w = torch.randn(5120, 1280, device=dev, dtype=torch.bfloat16)
        fn = lambda: gemm.linear_fwd(x, w)
    elif case == "gemm_relu2":
        x = torch.randn(16384, 1280, device=dev, dtype=torch.bfloat16)
        w = torch.randn(5120, 1280, device=dev, dtype=torch.bfloat16)
        fn = lambda: gemm.linear_relu2_fwd(x, w)
    elif case == "gemm_dw":
        dy = torch.randn(16384, 5120, device=dev, dtype=torch.bfloat16)
        x = torch.randn(16384, 1280, device=dev, dtype=torch.bfloat16)
        g = torch.zeros(5120, 1280, device=dev)
        fn = lambda: gemm.linear_dw(dy, x, g)
    else:
        B, T, H, D = 4, 2048, 10, 128
        M = B * T
        q, k, v, do = (torch.randn(M, H * D, device=dev, dtype=torch.bfloat16) for _ in range(4))
        o, lse = flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)
        fn = (lambda: flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)) if case == "fa_fwd" else \
            (lambda: flash_bwd(q, k, v, o, do, lse, B, T, H, D, D ** -0.5, True))
    for _ in range(4):
        fn()
    torch.cuda.synchronize(dev)


def trace_fa_fwd(dev, B: int = 16, T: int = 2048, H: int = 10, D: int = 128) -> dict:
    """Phase timeline (SM clock cycles) of CTA 0 of the two-tile flash-attention forward."""
    from ..ops._ext import C
    from ..ops.flash_attention import flash_fwd
    M = B * T
    q, k, v = (torch.randn(M, H * D, device=dev, dtype=torch.bfloat16) for _ in range(3))
    for _ in range(3):
        flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)
    buf = torch.zeros(4 * 64 * 8, dtype=torch.int64, device=dev)
    C().fa_trace_set(buf)
    flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)
    torch.cuda.synchronize(dev)
    C().fa_trace_set(None)
    t = buf.view(4, 64, 8).cpu()
    t0 = int(t[t > 0].min())
    names = {0: ["step top", "PV0(j) issued", "S0(j+1) issued", "PV1(j) issued", "S1(j+1) issued"],
             1: ["loop top", "S ready", "P computed", "O rescaled", "P in TMEM"],
             2: ["loop top", "S ready", "P computed", "O rescaled", "P in TMEM"]}
    out = {}
    for r, role in enumerate(["mma", "softmax0", "softmax1"]):
        rows = []
        for i in range(64):
            ev = [int(x) for x in t[r, i, :len(names[r])]]
            if any(ev):
                rows.append({n: (e - t0 if e else None) for n, e in zip(names[r], ev)})
        out[role] = rows
    return out


def trace_fa_bwd(dev, B: int = 16, T: int = 2048, H: int = 10, D: int = 128) -> dict:
    """Phase timeline (SM clock cycles) of CTA 0 of the pipelined flash-attention backward:
    per query tile, when each role reached each phase (see ``fa_stamp`` in
    csrc/kernels/attention_sm100.cu).  For reading where the pipeline waits."""
    from ..ops._ext import C
    from ..ops.flash_attention import flash_bwd, flash_fwd
    M = B * T
    q, k, v, do = (torch.randn(M, H * D, device=dev, dtype=torch.bfloat16) for _ in range(4))
    o, lse = flash_fwd(q, k, v, B, T, H, D, D ** -0.5, True)
    for _ in range(3):
        flash_bwd(q, k, v, o, do, lse, B, T, H, D, D ** -0.5, True)
    buf = torch.zeros(4 * 64 * 8, dtype=torch.int64, device=dev)
    C().fa_trace_set(buf)
    flash_bwd(q, k, v, o, do, lse, B, T, H, D, D ** -0.5, True)
    torch.cuda.synchronize(dev)
    C().fa_trace_set(None)
    t = buf.view(4, 64, 8).cpu()
    t0 = int(t[t > 0].min())
    names = {0: ["dP issued", "P ready", "S(i+1) issued", "dS ready", "loop top", "dO landed", "dQ drained"],
             1: ["loop top", "S ready", "P in TMEM", "dP ready", "dS computed", "dS tile free", "dS stored"],
             2: ["loop top", "dQ ready", "dQ read"], 3: ["Q issued", "dO issued"]}
    roles = ["mma", "softmax", "drain", "producer"]
    out = {}
    for r, role in enumerate(roles):
        rows = []
        for i in range(64):
            ev = [int(x) for x in t[r, i, :len(names[r])]]
            if not any(ev):
                continue
            rows.append({n: (e - t0 if e else None) for n, e in zip(names[r], ev)})
        out[role] = rows
    return out


DG_PHASES = ["entry", "set-up done", "weight loads issued", "grid dependency resolved", "first stage landed",
             "last MMA issued", "sums of squares done", "MMAs complete", "partial tile stored",
             "cluster barrier 1", "rows reduced + stored", "cluster barrier 2"]


def bench_decode_gemm(dev, peaks, M: int = 32, reps: int = 50) -> list[dict]:
    """Decode-step linears of the d20 model (M = 32 rows) through the decode GEMM: per
    shape, the event-timed mean of `reps` back-to-back launches cycling over enough weight
    copies (> L2) that every launch streams its weights from HBM, with and without
    programmatic dependent launch, and the phase timeline (ns from CTA 0's entry) of the
    first and last CTA of one launch."""
    from ..ops._ext import C, err_word
    shapes = [("qkv", 3840, 1280, 4, True), ("attn proj", 1280, 1280, 1, False), ("fc", 5120, 1280, 2, True),
              ("mlp proj", 1280, 5120, 1, False), ("lm_head", 8192, 1280, 0, True)]
    err = err_word(dev)
    out = []
    for name, N, K, epi, norm in shapes:
        copies = max(2, (160 << 20) // (N * K * 2) + 1)
        ws = [(torch.randn(N, K, device=dev) * K ** -0.5).bfloat16() for _ in range(copies)]
        x = torch.randn(M, K, device=dev).bfloat16()
        r = torch.randn(M, N, device=dev).bfloat16()
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        epi_c = 1 if epi in (1, 4) else (2 if epi == 2 else 0)   # QKV shape timed with the residual epilogue

        def run(pdl, i):
            C().decode_gemm(x, ws[i % copies], y, epi_c, norm, r if epi_c == 1 else None, None, None, None, 0.0,
                            None, None, None, None, None, 0, 0, pdl, err)
        row = {"name": name, "N": N, "K": K, "weight_mb": N * K * 2 / 1e6}
        for pdl in (False, True):
            for i in range(5):
                run(pdl, i)
            torch.cuda.synchronize(dev)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for i in range(reps):
                run(pdl, i)
            e.record()
            torch.cuda.synchronize(dev)
            us = s.elapsed_time(e) * 1000 / reps
            key = "pdl" if pdl else "plain"
            row[f"us_{key}"] = us
            row[f"gbs_{key}"] = N * K * 2 / us / 1e3
            row[f"frac_hbm_{key}"] = row[f"gbs_{key}"] / peaks["hbm_gbs"]
        buf = torch.zeros(32, dtype=torch.int64, device=dev)
        C().decode_gemm_trace_set(buf)
        run(False, 0)
        torch.cuda.synchronize(dev)
        C().decode_gemm_trace_set(None)
        t = buf.cpu().tolist()
        t0 = t[0]
        row["timeline_first_cta"] = {p: (t[i] - t0 if t[i] else None) for i, p in enumerate(DG_PHASES)}
        row["timeline_last_cta"] = {p: (t[16 + i] - t0 if t[16 + i] else None) for i, p in enumerate(DG_PHASES)}
        out.append(row)
        del ws
    return out


def bench_decode_attention(dev, peaks, B: int = 32, H: int = 10, D: int = 128, L: int = 576, Tmax: int = 896,
                           reps: int = 50) -> list[dict]:
    """Split decode attention over a head-major KV cache (the decode step's layout) for a
    sweep of cache-length splits: event-timed mean of `reps` launches cycling over enough
    cache copies (> L2) that every launch streams K and V from HBM."""
    from ..ops._ext import C
    per = B * H * Tmax * D * 2 * 2
    copies = max(2, (200 << 20) // per + 1)
    caches = [(torch.randn(B, H, Tmax, D, device=dev).bfloat16(), torch.randn(B, H, Tmax, D, device=dev).bfloat16())
              for _ in range(copies)]
    q = torch.randn(B, H * D, device=dev).bfloat16()
    ln = torch.tensor([L], dtype=torch.int32, device=dev)
    out = torch.empty(B, H * D, device=dev, dtype=torch.bfloat16)
    rows = []
    for splits in (3, 5, 7, 10, 14, 16):
        ws = torch.zeros(B * H * splits * (D + 4), device=dev)
        cnt = torch.zeros(B * H, dtype=torch.int32, device=dev)

        def run(i):
            kc, vc = caches[i % copies]
            C().decode_attn_split(q, kc, vc, ln, H, D, D ** -0.5, out, ws, cnt, splits, False)
        for i in range(5):
            run(i)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(reps):
            run(i)
        e.record()
        torch.cuda.synchronize(dev)
        us = s.elapsed_time(e) * 1000 / reps
        gbs = B * H * L * D * 2 * 2 / us / 1e3
        rows.append({"splits": splits, "ctas": B * H * splits, "us": us, "gbs": gbs, "frac_hbm": gbs / peaks["hbm_gbs"]})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", nargs="?", default="gemm")
    ap.add_argument("--one", default="", help="run one small case: gemm | gemm_relu2 | gemm_dw | fa_fwd | fa_bwd")
    ap.add_argument("--json", default="")
    ap.add_argument("--trace", action="store_true", help="print the flash backward phase timeline of CTA 0")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    if args.one:
        one_kernel(args.one, dev)
        return
    if args.trace:
        tl = {"backward": trace_fa_bwd(dev), "forward": trace_fa_fwd(dev)}
        for kern, roles in tl.items():
            for role, rows in roles.items():
                print(f"== {kern} {role}")
                for i, r in enumerate(rows):
                    print(f"  {i:3d} " + "  ".join(f"{k}={v}" for k, v in r.items()))
        if args.json:
            with open(args.json, "w") as f:
                json.dump(tl, f, indent=1)
        return
    out = {"peaks": peaks}
    if args.what in ("gemm", "all"):
        out["gemm"] = bench_gemm(dev, peaks)
        for r in out["gemm"]:
            print(f"{r['name']:>20s}  {r['ms']:8.3f} ms  {r['tflops']:7.1f} TF/s ({r['frac_of_measured']:.2f} of "
                  f"{peaks['source']})   torch {r['torch_ms']:8.3f} ms {r['torch_tflops']:7.1f} TF/s")
    if args.what in ("decode", "all"):
        out["decode_gemm"] = bench_decode_gemm(dev, peaks)
        for r in out["decode_gemm"]:
            print(f"{r['name']:>12s} {r['weight_mb']:6.1f} MB  plain {r['us_plain']:6.2f} us ({r['frac_hbm_plain']:.2f} of HBM)"
                  f"  pdl {r['us_pdl']:6.2f} us ({r['frac_hbm_pdl']:.2f})")
            for cta in ("timeline_first_cta", "timeline_last_cta"):
                print(f"   {cta}: " + ", ".join(f"{k}={v}" for k, v in r[cta].items()))
        out["decode_attention"] = bench_decode_attention(dev, peaks)
        for r in out["decode_attention"]:
            print(f"  decode attention splits {r['splits']:2d} ({r['ctas']} CTAs): {r['us']:6.2f} us "
                  f"{r['gbs']:7.1f} GB/s ({r['frac_hbm']:.2f} of HBM)")
    if args.what in ("attn", "all"):
        out["attention"] = bench_attention(dev, peaks)
        for r in out["attention"]:
            print(f"{r['name']:>20s}  {r['ms']:8.3f} ms  {r['tflops']:7.1f} TF/s ({r['frac_of_measured']:.2f} of "
                  f"{peaks['source']})   torch sdpa {r['torch_sdpa_ms']:.3f} ms {r['torch_sdpa_tflops']:7.1f} TF/s")
    from ..ops._ext import check_errors
    check_errors(dev)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
