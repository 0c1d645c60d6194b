"""KV-cache greedy decoding for the plain GPT family (new: the reference has none).

``Generator(model).generate(prompts, max_new_tokens)``:

* prefill: the prompt runs through the training kernels (fused mix+norm, tcgen05
  GEMMs, RoPE+QK-norm, tcgen05 flash attention) in one pass; every layer's normalised
  keys and values land in a ``[B, T_max, H*D]`` cache (the projection buffer's own
  layout, so the copy is a strided row copy);
* decode: one token per sequence per step, five launches per block through the
  decode GEMM (``csrc/kernels/decode_gemm.cu``: swapped-operand tcgen05 tiles, split-K
  over a thread-block cluster reduced in distributed shared memory, programmatic
  dependent launch so each kernel's weight stream starts under the previous kernel):
    1. QKV projection of the mixed residual with its RMS norm folded in (row scale),
       RoPE + QK-norm at the device-side position, k / v rows written into the cache;
    2. split single-query attention over the cache;
    3. attention projection + residual;
    4. MLP up-projection with the RMS norm folded in, relu^2;
    5. MLP down-projection + residual, then the next block's residual mix
       (lambda_r x + lambda_0 x0), so the next QKV projection reads it directly;
  then the lm_head with the final norm folded in and a greedy argmax (argmax of the
  softcapped logits = argmax of the raw ones).  Position and length live in device
  memory and the argmax feeds the next step's input in device memory, so the whole step
  is captured once in a CUDA graph and replayed.  Every buffer of the step is allocated
  once, up front; the KV caches are head-major ([B, H, T_max, D]) so each (sequence,
  head) of the decode attention streams one contiguous range.

``generate_reference`` recomputes the full forward for every new token; it is the
oracle the cached path is tested against and the path for non-plain members.

The reference has no generation path; its forward (``GPT.forward``, ``train.py:3412-3485``)
is what prefill and the oracle reproduce.
"""
from __future__ import annotations

import os

import torch

from ..ops import gemm
from ..ops._ext import C, err_word

# epilogues of the decode GEMM (csrc/kernels/decode_gemm.cu)
DEC_PLAIN, DEC_RES, DEC_RELU2, DEC_MIX, DEC_QKV = 0, 1, 2, 3, 4
from ..ops.flash_attention import flash_fwd, supported
from ..ops.fused import w16


def _is_plain(model) -> bool:
    rc = model.rc
    return not (rc.ve or rc.ngram_ve or rc.local_conv or rc.qk_shift or rc.head_gate or rc.out_pool or
                rc.x0_gate or rc.mlp_sandwich_norm or rc.gated_mlp or rc.coalesced_swiglu or rc.doc_mask or
                rc.out_bigram or rc.engram or rc.parallel_block or rc.block_nudge or rc.selective_gate or
                "S" in rc.window_pattern or (model.config.n_kv_heads not in (0, model.config.n_head)))


@torch.no_grad()
def generate_reference(model, prompts: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
    """Greedy decoding by full recomputation (no cache)."""
    idx = prompts
    out = []
    for _ in range(max_new_tokens):
        logits = model(idx)[:, -1]
        nxt = logits.argmax(-1)
        out.append(nxt)
        idx = torch.cat([idx, nxt[:, None].to(idx.dtype)], dim=1)
    return torch.stack(out, 1)


class Generator:
    def __init__(self, model, max_batch: int, max_len: int):
        if not _is_plain(model):
            raise NotImplementedError("the cached decoder serves the plain member of the family; "
                                      "use generate_reference for the others")
        self.m = model
        cfg = model.config
        self.dev = model.get_device()
        self.B = max_batch
        self.Tmax = max_len
        self.H, self.D, self.Cd = cfg.n_head, cfg.head_dim, cfg.n_embd
        self.V, self.Vp = cfg.vocab_size, cfg.padded_vocab_size
        self.scale = cfg.attn_scale if cfg.attn_scale > 0 else self.D ** -0.5
        L = cfg.n_layer
        dev = self.dev
        bf = torch.bfloat16
        # head_dim 128 (the fused decode step): head-major caches [B, H, T_max, D], so each
        # (sequence, head) of the decode attention reads one contiguous stream; otherwise
        # the projection buffer's token-major layout [B, T_max, H*D]
        self.fused_decode = self.D == 128 and self.B <= 128
        # programmatic dependent launch of the decode kernels (TFB_DECODE_PDL=0 turns it off)
        self.pdl = os.environ.get("TFB_DECODE_PDL", "1") != "0"
        shape = (self.B, self.H, self.Tmax, self.D) if self.fused_decode else (self.B, self.Tmax, self.Cd)
        self.kc = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(L)]
        self.vc = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(L)]
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)  # [position, cache length]
        self.idx = torch.zeros(self.B, 1, dtype=torch.int32, device=dev)
        self.graph = None
        self.tokens = None
        self.ws: dict = {}   # decode GEMM workspaces (zeroed fp32 sums + counters) per shape
        # cache-length splits of the decode attention, one per 128 cache rows (at most 16).
        # In isolation 3 splits (one wave) ran faster at batch 32 x 10 heads x 576 keys
        # (22.7 vs 26.7 us, utils/kernel_bench.py decode), but inside the decode step, where
        # the next projection's CTAs launch early, 7 splits gave the faster step
        self.att_splits = max(1, min(16, self.Tmax // 128))
        self.att_ws = torch.zeros(self.B * self.H * self.att_splits * (self.D + 4), dtype=torch.float32, device=dev)
        self.att_cnt = torch.zeros(self.B * self.H, dtype=torch.int32, device=dev)
        blocks = list(model.transformer.h)
        self.wqkv = [torch.cat([w16(b.attn.c_q.weight), w16(b.attn.c_k.weight), w16(b.attn.c_v.weight)], 0).contiguous()
                     for b in blocks]
        self.wo = [w16(b.attn.c_proj.weight) for b in blocks]
        self.wfc = [w16(b.mlp.c_fc.weight) for b in blocks]
        self.wp = [w16(b.mlp.c_proj.weight) for b in blocks]
        self.lam = [(b.resid_lambda.detach(), b.x0_lambda.detach()) for b in blocks]
        self.wlm = w16(model.lm_head.weight)
        self.wte = model.transformer.wte.weight.detach()
        self.tau = model.rc.relu2_tau
        cos, sin = model.cos, model.sin
        self.cos = cos.reshape(-1, cos.shape[-1]).to(bf).contiguous()
        self.sin = sin.reshape(-1, sin.shape[-1]).to(bf).contiguous()
        # decode-step buffers (fixed addresses: the step is captured in a CUDA graph)
        Bm, Cd = self.B, self.Cd
        self.d_x0 = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_xm = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_h = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_rstd = torch.empty(Bm, dtype=torch.float32, device=dev)
        self.d_q = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_y = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_x = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_act = torch.empty(Bm, self.wfc[0].shape[0], dtype=bf, device=dev)
        self.d_xf = torch.empty(Bm, Cd, dtype=bf, device=dev)
        self.d_logits = torch.empty(Bm, self.wlm.shape[0], dtype=bf, device=dev)

    # ------------------------------------------------------------------ prefill
    def _block_rows(self, i, x, x0, M, T, pos_t=None, prefill=True):
        Cd, H, D = self.Cd, self.H, self.D
        xm = torch.empty_like(x)
        h = torch.empty_like(x)
        rstd = torch.empty(M, dtype=torch.float32, device=self.dev)
        C().mix_norm_fwd(x, x0, self.lam[i][0], self.lam[i][1], xm, h, rstd)
        qkv = gemm.linear_fwd(h, self.wqkv[i]) if prefill else gemm.linear_decode(h, self.wqkv[i], self.ws)
        qkn = torch.empty((M, 2 * Cd), dtype=torch.bfloat16, device=self.dev)
        C().rope_norm_fwd(qkv, 0, 2 * H, D, self.cos, self.sin, T, 0, None, qkn, pos_t)
        if prefill:
            B = M // T
            if self.fused_decode:
                self.kc[i][:B, :, :T].copy_(qkn[:, Cd:].view(B, T, H, D).transpose(1, 2))
                self.vc[i][:B, :, :T].copy_(qkv[:, 2 * Cd:].view(B, T, H, D).transpose(1, 2))
            else:
                self.kc[i][:B, :T].copy_(qkn[:, Cd:].view(B, T, Cd))
                self.vc[i][:B, :T].copy_(qkv[:, 2 * Cd:].view(B, T, Cd))
            y, _ = flash_fwd(qkn[:, :Cd], qkn[:, Cd:], qkv[:, 2 * Cd:], B, T, H, D, self.scale, True)
        else:
            C().kv_append(qkn[:, Cd:], qkv[:, 2 * Cd:], self.kc[i], self.vc[i], self.counters[0:1])
            y = torch.empty((M, Cd), dtype=torch.bfloat16, device=self.dev)
            if D == 128:   # cache length split over several CTAs per (batch, head)
                C().decode_attn_split(qkn[:, :Cd], self.kc[i], self.vc[i], self.counters[1:2], H, D, self.scale, y,
                                      self.att_ws, self.att_cnt, self.att_splits, False)
            else:
                C().decode_attn(qkn[:, :Cd], self.kc[i], self.vc[i], self.counters[1:2], H, D, self.scale, y)
        if prefill:
            x = gemm.linear_fwd(y, self.wo[i], residual=xm)
            h2 = torch.empty_like(x)
            C().rmsnorm_fwd(x, h2, None)
            act, _ = gemm.linear_relu2_fwd(h2, self.wfc[i], tau=self.tau)
            return gemm.linear_fwd(act, self.wp[i], residual=x)
        # decode: a few rows per step -> one split-K GEMM launch each (epilogue fused)
        x = gemm.linear_decode(y, self.wo[i], self.ws, residual=xm)
        h2 = torch.empty_like(x)
        C().rmsnorm_fwd(x, h2, None)
        act = gemm.linear_decode(h2, self.wfc[i], self.ws, relu2=True, tau=self.tau)
        return gemm.linear_decode(act, self.wp[i], self.ws, residual=x)

    def _head(self, x):
        xf = torch.empty_like(x)
        C().rmsnorm_fwd(x, xf, None)
        if x.shape[0] <= 64:
            return gemm.linear_decode(xf, self.wlm, self.ws)
        return gemm.linear_fwd(xf, self.wlm)

    def _embed(self, idx):
        B, T = idx.shape
        out = torch.empty((B * T, self.Cd), dtype=torch.bfloat16, device=self.dev)
        rstd = torch.empty(B * T, dtype=torch.float32, device=self.dev)
        C().embed_norm_fwd(idx, self.wte, out, rstd)
        return out

    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor) -> torch.Tensor:
        B, T = prompts.shape
        assert B <= self.B and T < self.Tmax and supported(T, self.D)
        idx = prompts.to(device=self.dev, dtype=torch.int32).contiguous()
        x0 = self._embed(idx)
        x = x0
        for i in range(len(self.wqkv)):
            x = self._block_rows(i, x, x0, B * T, T)
        last = x.view(B, T, self.Cd)[:, -1].contiguous()
        logits = self._head(last)
        self.counters.copy_(torch.tensor([T, T + 1], dtype=torch.int32))
        C().argmax_rows(logits, self.V, self.idx, None, self.counters, T)
        return logits

    # ------------------------------------------------------------------ decode
    def _decode_step(self):
        if not self.fused_decode:
            x0 = self._embed(self.idx)
            x = x0
            for i in range(len(self.wqkv)):
                x = self._block_rows(i, x, x0, self.B, 1, pos_t=self.counters[0:1], prefill=False)
            logits = self._head(x)
        else:
            logits = self._fused_step()
        C().argmax_rows(logits, self.V, self.idx, self.tokens, self.counters, self.start)
        C().step_advance(self.counters)

    def _fused_step(self):
        """One decode step of the plain member with head_dim 128 through the decode GEMM:
        five launches per block (see the module docstring)."""
        c = C()
        err = err_word(self.dev)
        x0, xm, q, y, x, act, xf = self.d_x0, self.d_xm, self.d_q, self.d_y, self.d_x, self.d_act, self.d_xf
        c.embed_norm_fwd(self.idx, self.wte, x0, self.d_rstd)
        lr, l0 = self.lam[0]
        c.mix_norm_fwd(x0, x0, lr, l0, xm, self.d_h, self.d_rstd)   # block 0's mix: x = x0
        pos, ln = self.counters[0:1], self.counters[1:2]
        L = len(self.wqkv)
        for i in range(L):
            c.decode_gemm(xm, self.wqkv[i], q, DEC_QKV, True, None, None, None, None, 0.0, self.cos, self.sin,
                          pos, self.kc[i], self.vc[i], self.H, 0, self.pdl, err)
            c.decode_attn_split(q, self.kc[i], self.vc[i], ln, self.H, self.D, self.scale, y, self.att_ws,
                                self.att_cnt, self.att_splits, self.pdl)
            c.decode_gemm(y, self.wo[i], x, DEC_RES, False, xm, None, None, None, 0.0, None, None, None, None, None,
                          0, 0, self.pdl, err)
            c.decode_gemm(x, self.wfc[i], act, DEC_RELU2, True, None, None, None, None, float(self.tau), None, None,
                          None, None, None, 0, 0, self.pdl, err)
            if i + 1 < L:
                nr, n0 = self.lam[i + 1]
                c.decode_gemm(act, self.wp[i], xm, DEC_MIX, False, x, x0, nr, n0, 0.0, None, None, None, None, None,
                              0, 0, self.pdl, err)
            else:
                c.decode_gemm(act, self.wp[i], xf, DEC_RES, False, x, None, None, None, 0.0, None, None, None, None,
                              None, 0, 0, self.pdl, err)
        c.decode_gemm(xf, self.wlm, self.d_logits, DEC_PLAIN, True, None, None, None, None, 0.0, None, None, None,
                      None, None, 0, 0, self.pdl, err)
        return self.d_logits

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        B, T = prompts.shape
        assert B == self.B, "a generator is built for a fixed batch"
        assert T + max_new_tokens <= self.Tmax
        self.tokens = torch.zeros(B, max_new_tokens, dtype=torch.int32, device=self.dev)
        self.start = T
        self.prefill(prompts)
        # the first new token comes from the prefill's last position
        self.tokens[:, 0] = self.idx[:, 0]
        self.counters.copy_(torch.tensor([T, T + 1], dtype=torch.int32))
        self.start = T - 1  # slot = position - start: position T produces token 1
        n = max_new_tokens - 1
        if n <= 0:
            return self.tokens
        if use_graph:
            self._decode_step()            # warm-up (also sets every TMA descriptor)
            self._rewind(T)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._decode_step()
            self.graph = g
            self._rewind(T)
            for _ in range(n):
                g.replay()
        else:
            for _ in range(n):
                self._decode_step()
        return self.tokens

    @torch.no_grad()
    def replay_steps(self, n: int, T: int) -> None:
        """Replays the captured decode step n times from position T (after ``generate``),
        for timing and profiling one step in isolation."""
        assert self.graph is not None, "generate(..., use_graph=True) captures the step first"
        self._rewind(T)
        for _ in range(n):
            self.graph.replay()

    def _rewind(self, T):
        self.counters.copy_(torch.tensor([T, T + 1], dtype=torch.int32, device=self.dev))
        self.idx[:, 0] = self.tokens[:, 0]
