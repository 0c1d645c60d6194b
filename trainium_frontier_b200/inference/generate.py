"""KV-cache greedy decoding for the plain GPT family (new: the reference has none).

``Generator(model).generate(prompts, max_new_tokens)``:

* prefill: the prompt runs through the training kernels (fused mix+norm, tcgen05
  GEMMs, RoPE+QK-norm, tcgen05 flash attention) in one pass; every layer's normalised
  keys and values land in a ``[B, T_max, H*D]`` cache (the projection buffer's own
  layout, so the copy is a strided row copy);
* decode: one token per sequence per step -- mix+norm -> QKV GEMM -> RoPE+QK-norm at
  the device-side position -> cache append -> single-query attention over the cache
  -> projection + residual -> norm -> relu^2 MLP -> final norm -> lm_head -> greedy
  argmax (argmax of the softcapped logits = argmax of the raw ones).  Position and
  length live in device memory and the argmax feeds the next step's input in device
  memory, so the whole step is captured once in a CUDA graph and replayed.

``generate_reference`` recomputes the full forward for every new token; it is the
oracle the cached path is tested against and the path for non-plain members.

The reference has no generation path; its forward (``GPT.forward``, ``train.py:3412-3485``)
is what prefill and the oracle reproduce.
"""
from __future__ import annotations

import torch

from ..ops import gemm
from ..ops._ext import C, err_word
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
        self.kc = [torch.zeros(self.B, self.Tmax, self.Cd, dtype=bf, device=dev) for _ in range(L)]
        self.vc = [torch.zeros(self.B, self.Tmax, self.Cd, dtype=bf, device=dev) for _ in range(L)]
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)  # [position, cache length]
        self.idx = torch.zeros(self.B, 1, dtype=torch.int32, device=dev)
        self.graph = None
        self.tokens = None
        self.ws: dict = {}   # decode GEMM workspaces (zeroed fp32 sums + counters) per shape
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
            self.kc[i][:B, :T].copy_(qkn[:, Cd:].view(B, T, Cd))
            self.vc[i][:B, :T].copy_(qkv[:, 2 * Cd:].view(B, T, Cd))
            y, _ = flash_fwd(qkn[:, :Cd], qkn[:, Cd:], qkv[:, 2 * Cd:], B, T, H, D, self.scale, True)
        else:
            C().kv_append(qkn[:, Cd:], qkv[:, 2 * Cd:], self.kc[i], self.vc[i], self.counters[0:1])
            y = torch.empty((M, Cd), dtype=torch.bfloat16, device=self.dev)
            if D == 128:   # cache length split over several CTAs per (batch, head)
                C().decode_attn_split(qkn[:, :Cd], self.kc[i], self.vc[i], self.counters[1:2], H, D, self.scale, y,
                                      self.att_ws, self.att_cnt, self.att_splits)
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
        x0 = self._embed(self.idx)
        x = x0
        for i in range(len(self.wqkv)):
            x = self._block_rows(i, x, x0, self.B, 1, pos_t=self.counters[0:1], prefill=False)
        logits = self._head(x)
        C().argmax_rows(logits, self.V, self.idx, self.tokens, self.counters, self.start)
        C().step_advance(self.counters)

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
