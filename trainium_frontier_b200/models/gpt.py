"""The GPT family (reference ``train.py:1407-1433``, ``train.py:2237-3485``).

Plain member (default): untied ``wte``/``lm_head`` with vocab padded to a multiple of
64; the embedding is RMS-normed and kept as ``x0``; each block mixes
``x <- resid_lambda * x + x0_lambda * x0`` (learned per-block scalars), then pre-norm
attention (RoPE followed by parameter-free QK RMSNorm, causal) and a relu^2 MLP; final
norm, ``lm_head``, logit softcap ``S tanh(z / S)``.

Module and parameter names are the reference's, so ``state_dict`` keys -- and therefore
the ``out/final.pt`` payload -- are interchangeable (``transformer.wte.weight``,
``transformer.h.{i}.attn.c_q.weight``, ..., ``transformer.h.{i}.resid_lambda``,
``lm_head.weight``, ``value_embeds.{i}.weight``, ``ngram_embeds.b{i}.weight``).

Optional members of the family, all off by default and all step-0 no-ops where the
reference's are: value embeddings with input gates (``ve``), hashed bigram/trigram
value embeddings (``ngram_ve``), depthwise causal conv (``local_conv``), causal Q/K
token shift (``qk_shift``), per-head output gate (``head_gate``), output pooling of the
last layers (``out_pool``), input-dependent x0 gate (``x0_gate``), MLP sandwich norm,
shifted relu^2 (``relu2_tau``), gated / SwiGLU MLP, GQA (``n_kv_heads``), explicit
attention scale, document masking and sliding-window layers, the output bigram table
(``out_bigram``).

Hot path: on CUDA with the plain configuration each block is five fused kernels plus
attention: [mix + norm] -> [QKV GEMM] -> [RoPE + QK-norm + attention] -> [proj GEMM +
residual] -> [norm] -> [fc GEMM + relu^2] -> [proj GEMM + residual].
"""
from __future__ import annotations

import math
from dataclasses import asdict

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import GPTConfig, RunConfig, parse_int_tuple


class Linear(nn.Linear):
    """Bias-free linear whose forward runs through ``ops.linear`` (the fp32 weight is
    cast to the compute dtype; on the GPU a cached bf16 copy is used)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__(in_features, out_features, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(x, self.weight)


class CausalConv(nn.Module):
    """Depthwise causal conv1d with K-1 left padding, zero-init (train.py:1316-1329)."""

    def __init__(self, channels: int, kernel: int):
        super().__init__()
        self.kernel = kernel
        self.weight = nn.Parameter(torch.zeros(channels, 1, kernel))

    def forward(self, x: torch.Tensor) -> torch.Tensor:  # [B, T, C]
        return ops.causal_conv(x, self.weight)


def causal_shift_1(x: torch.Tensor) -> torch.Tensor:
    return F.pad(x[:, :-1], (0, 0, 1, 0))


def has_ve(layer_idx: int, n_layer: int) -> bool:
    """Value embeddings on alternating layers, always including the last."""
    return layer_idx % 2 == (n_layer - 1) % 2


def _ngram_layers(spec: str, n_layer: int) -> set[int]:
    if not spec:
        return {i for i in range(n_layer) if has_ve(i, n_layer)}
    out = set()
    for v in parse_int_tuple(spec):
        out.add(v % n_layer)
    return out


def _next_prime(n: int) -> int:
    def is_prime(k):
        if k < 2:
            return False
        if k % 2 == 0:
            return k == 2
        r = int(k ** 0.5)
        for d in range(3, r + 1, 2):
            if k % d == 0:
                return False
        return True
    while not is_prime(n):
        n += 1
    return n


def _largest_prime_below(n: int) -> int:
    k = n
    while k > 2:
        if all(k % d for d in range(2, int(k ** 0.5) + 1)):
            return k
        k -= 1
    return 2


def _ngram_primes(layer_idx: int) -> tuple[int, int, int]:
    """Layer-dependent multipliers, bounded so id * p fits int32 for ids < 2^14."""
    base = 1000 + 97 * layer_idx
    p1 = _next_prime(base * 31 + 7)
    p2 = _next_prime(base * 53 + 11)
    p3 = _next_prime(base * 71 + 13)
    return p1, p2, p3


class CausalSelfAttention(nn.Module):
    def __init__(self, config: GPTConfig, rc: RunConfig, layer_idx: int):
        super().__init__()
        self.n_head = config.n_head
        self.n_embd = config.n_embd
        self.head_dim = config.n_embd // config.n_head
        self.n_kv_heads = config.n_kv_heads or config.n_head
        if self.n_head % self.n_kv_heads:
            raise ValueError("n_kv_heads must divide n_head")
        self.kv_repeat = self.n_head // self.n_kv_heads
        self.c_q = Linear(config.n_embd, config.n_embd)
        self.c_k = Linear(config.n_embd, self.n_kv_heads * self.head_dim)
        self.c_v = Linear(config.n_embd, self.n_kv_heads * self.head_dim)
        self.c_proj = Linear(config.n_embd, config.n_embd)
        self.attn_scale = config.attn_scale if config.attn_scale > 0.0 else None
        gc = rc.ve_gate_channels
        self.gate_channels = gc
        self.ve_gate = Linear(gc, self.n_head) if (rc.ve and has_ve(layer_idx, config.n_layer)) else None
        ng = rc.ngram_ve and layer_idx in _ngram_layers(rc.ngram_ve_layers, config.n_layer)
        self.ve_gate_bi = Linear(gc, self.n_head) if ng else None
        self.ve_gate_tri = Linear(gc, self.n_head) if (ng and rc.ngram_ve_trigram) else None
        if rc.head_gate:
            lo = min(3 * gc, max(0, config.n_embd - rc.head_gate_channels))
            self.head_gate_lo, self.head_gate_hi = lo, lo + rc.head_gate_channels
            self.head_gate = Linear(rc.head_gate_channels, self.n_head)
            self.head_gate_bias = nn.Parameter(torch.full((self.n_head,), float(rc.head_gate_bias)))
        else:
            self.head_gate = None
        self.head_gate_norm = rc.head_gate_norm
        self.head_gate_mul = rc.head_gate_mul

    @property
    def plain(self) -> bool:
        return (self.ve_gate is None and self.ve_gate_bi is None and self.ve_gate_tri is None
                and self.head_gate is None and self.kv_repeat == 1)

    def forward(self, x_q, x_k, x_v, ve, cos, sin, attn_mask, ve_bi=None, ve_tri=None):
        b, t, c = x_q.shape
        if self.plain and attn_mask is None and x_q is x_k and x_k is x_v:
            return ops.qkv_attention(x_q, [self.c_q.weight, self.c_k.weight, self.c_v.weight], cos, sin,
                                     self.n_head, self.head_dim, self.attn_scale)  # c_proj: by the block
        q = ops.linear(x_q, self.c_q.weight).view(b, t, self.n_head, self.head_dim)
        k = ops.linear(x_k, self.c_k.weight).view(b, t, self.n_kv_heads, self.head_dim)
        v = ops.linear(x_v, self.c_v.weight).view(b, t, self.n_kv_heads, self.head_dim)
        if self.kv_repeat > 1:
            k = k.repeat_interleave(self.kv_repeat, dim=2).contiguous()
            v = v.repeat_interleave(self.kv_repeat, dim=2).contiguous()
        gc = self.gate_channels
        if ve is not None:
            gate = 2 * torch.sigmoid(ops.linear(x_v[..., :gc], self.ve_gate.weight))
            v = v + gate.unsqueeze(-1) * ve.view(b, t, self.n_head, self.head_dim)
        if ve_bi is not None:
            g_bi = 2 * torch.sigmoid(ops.linear(x_v[..., gc:2 * gc], self.ve_gate_bi.weight))
            v = v + g_bi.unsqueeze(-1) * ve_bi.view(b, t, self.n_head, self.head_dim)
        if ve_tri is not None:
            g_tri = 2 * torch.sigmoid(ops.linear(x_v[..., 2 * gc:3 * gc], self.ve_gate_tri.weight))
            v = v + g_tri.unsqueeze(-1) * ve_tri.view(b, t, self.n_head, self.head_dim)
        q = ops.rope_norm(q, cos, sin)
        k = ops.rope_norm(k, cos, sin)
        y = ops.attention(q, k, v, causal=attn_mask is None, scale=self.attn_scale,
                          attn_mask=None if attn_mask is None else attn_mask[..., :t, :t].to(q.dtype))
        y = y.reshape(b, t, c)
        if self.head_gate is not None:
            yh = y.view(b, t, self.n_head, self.head_dim)
            if self.head_gate_norm:
                yh = ops.norm(yh)
            g = ops.linear(x_q[..., self.head_gate_lo:self.head_gate_hi], self.head_gate.weight)
            g = self.head_gate_mul * torch.sigmoid(g + self.head_gate_bias.to(g.dtype))
            y = (yh * g.unsqueeze(-1)).view(b, t, c)
        return y


class MLP(nn.Module):
    def __init__(self, config: GPTConfig, rc: RunConfig):
        super().__init__()
        hidden = config.mlp_ratio * config.n_embd
        self.swiglu_hidden = 0
        if rc.coalesced_swiglu:
            if rc.coalesced_swiglu_hidden > 0:
                self.swiglu_hidden = int(rc.coalesced_swiglu_hidden)
            else:
                exact = (2.0 / 3.0) * config.mlp_ratio * config.n_embd
                self.swiglu_hidden = max(128, int(round(exact / 128.0)) * 128)
            hidden = self.swiglu_hidden
        fc_out = 2 * hidden if self.swiglu_hidden else hidden
        self.c_fc = Linear(config.n_embd, fc_out)
        self.c_gate = Linear(config.n_embd, hidden) if rc.gated_mlp else None
        self.c_proj = Linear(hidden, config.n_embd)
        self.tau = rc.relu2_tau

    @property
    def plain(self) -> bool:
        return not self.swiglu_hidden and self.c_gate is None

    def forward(self, x, residual=None):
        if self.plain:
            return ops.mlp_relu2(x, self.c_fc.weight, self.c_proj.weight, residual, self.tau)
        h = ops.linear(x, self.c_fc.weight)
        if self.swiglu_hidden:
            a = F.silu(h[..., :self.swiglu_hidden]) * h[..., self.swiglu_hidden:]
        else:
            a = h * F.silu(ops.linear(x, self.c_gate.weight))
        return ops.linear(a, self.c_proj.weight, residual)


ENGRAM_HASH_PRIMES = tuple(_next_prime(20011 + 7919 * k) for k in range(24))


def engram_primes(head_idx: int, order: int) -> tuple[int, ...]:
    """Multipliers of one Engram hash head (oldest token first); orders use disjoint
    12-prime regions so heads of order 2 and 3 never share one (train.py:1182-1206)."""
    base = (order - 2) * 12 + head_idx * order
    if base + order > len(ENGRAM_HASH_PRIMES):
        raise ValueError("too many Engram hash heads for the prime table")
    return tuple(ENGRAM_HASH_PRIMES[base + j] for j in range(order))


def _rng_neutral(build):
    """Build a module without moving the CPU generator (its weights are overwritten by
    init_weights, so construction must not shift any later tensor's initial values)."""
    state = torch.random.get_rng_state()
    try:
        return build()
    finally:
        torch.random.set_rng_state(state)


class EngramLite(nn.Module):
    """Hashed n-gram memory read through a hidden-state gate (train.py:2767-2840):
    Y = SiLU(conv(norm(a v))) + a v with a = sigmoid(<norm q, norm k> / sqrt(d)),
    k = W_K e, v = W_V e, q = W_Q h (or h), e = the gathered table rows of the current
    token's 2-/3-gram hashes.  Zero tables and a zero conv make it an exact no-op at
    step 0 while W_K / W_V stay nonzero so the tables receive gradient."""

    def __init__(self, config: GPTConfig, rc: RunConfig, padded_vocab: int, share_e_dim: int | None = None):
        super().__init__()
        self.orders = tuple(int(o) for o in rc.engram_orders.split(",") if o.strip())
        self.heads = rc.engram_heads
        self.share = share_e_dim is not None
        self.mem_dim = rc.engram_mem_dim
        self.rows = rc.engram_table_mult * padded_vocab
        self.mod = _largest_prime_below(self.rows)
        dt = torch.bfloat16 if rc.engram_bf16 else torch.float32
        self.table_keys = tuple(f"e{h}o{o}" for o in self.orders for h in range(self.heads))
        if self.share:
            self.tables = nn.ModuleDict()
            self.e_dim = share_e_dim
        else:
            self.tables = nn.ModuleDict({k: nn.Embedding(self.rows, self.mem_dim,
                                                         _weight=torch.zeros(self.rows, self.mem_dim, dtype=dt))
                                         for k in self.table_keys})
            self.e_dim = self.mem_dim * len(self.table_keys)
        self.key_dim = rc.engram_key_dim if rc.engram_key_dim > 0 else config.n_embd
        self.w_k = _rng_neutral(lambda: Linear(self.e_dim, self.key_dim))
        self.w_v = _rng_neutral(lambda: Linear(self.e_dim, config.n_embd))
        self.w_q = _rng_neutral(lambda: Linear(config.n_embd, self.key_dim)) if self.key_dim != config.n_embd else None
        self.conv = CausalConv(config.n_embd, rc.engram_conv_kernel) if rc.engram_conv_kernel > 0 else None
        self.scale = self.key_dim ** -0.5

    def gather(self, idx: dict[str, torch.Tensor], dtype: torch.dtype) -> torch.Tensor:
        parts = [self.tables[k].weight[idx[k]].to(dtype) for k in self.table_keys]
        return parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)

    def forward(self, h: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
        k = ops.linear(e, self.w_k.weight)
        v = ops.linear(e, self.w_v.weight)
        q = ops.linear(h, self.w_q.weight) if self.w_q is not None else h
        a = torch.sigmoid((ops.norm(q) * ops.norm(k)).sum(dim=-1, keepdim=True) * self.scale)
        vt = a * v
        if self.conv is None:
            return vt
        return F.silu(self.conv(ops.norm(vt))) + vt


class Block(nn.Module):
    def __init__(self, config: GPTConfig, rc: RunConfig, layer_idx: int):
        super().__init__()
        self.attn = CausalSelfAttention(config, rc, layer_idx)
        self.mlp = MLP(config, rc)
        self.resid_lambda = nn.Parameter(torch.ones(1))
        self.x0_lambda = nn.Parameter(torch.zeros(1))
        self.x0_gate_s = nn.Parameter(torch.zeros(1)) if rc.x0_gate else None
        self.local_conv = CausalConv(config.n_embd, rc.local_conv_kernel) if rc.local_conv else None
        self.qk_shift_beta = (nn.Parameter(torch.full((config.n_embd,), float(rc.qk_shift_beta)),
                                           requires_grad=not rc.qk_shift_freeze) if rc.qk_shift else None)
        self.sandwich = rc.mlp_sandwich_norm
        # parallel block: attention and MLP read the same normed residual (train.py:2708-2746)
        if rc.parallel_block:
            self.par_lambda_a = nn.Parameter(torch.ones(1))
            self.par_lambda_m = nn.Parameter(torch.ones(1))
        else:
            self.par_lambda_a = self.par_lambda_m = None
        # frozen zero nudge: an exact identity kept out of every optimizer group
        self.block_nudge = nn.Parameter(torch.zeros(1), requires_grad=False) if rc.block_nudge else None
        self.nudge_site = rc.block_nudge_site
        # data-dependent resid / x0 mix from the first channels (zero-init => static lambdas)
        self.gate_channels = rc.selective_gate_channels
        self.scalar_gate = Linear(rc.selective_gate_channels, 2) if rc.selective_gate else None

    @property
    def plain(self) -> bool:
        return (self.x0_gate_s is None and self.local_conv is None and self.qk_shift_beta is None
                and not self.sandwich and self.attn.plain and self.mlp.plain and self.par_lambda_a is None
                and self.block_nudge is None and self.scalar_gate is None)

    def forward(self, x, x0, ve, cos, sin, attn_mask, ve_bi=None, ve_tri=None):
        tpc = getattr(self, "_tpc", None)
        if tpc is not None:
            from ..parallel.tensor_parallel import block_forward_tp
            return block_forward_tp(self, x, x0, cos, sin, tpc, self._layer_idx)
        fast = (self.x0_gate_s is None and self.local_conv is None and self.qk_shift_beta is None
                and not self.sandwich and attn_mask is None and self.attn.plain and self.par_lambda_a is None
                and self.block_nudge is None and self.scalar_gate is None)
        if fast:
            xm, h = ops.mix_norm(x, x0, self.resid_lambda, self.x0_lambda)
            y = self.attn(h, h, h, None, cos, sin, None)
            x = ops.linear(y, self.attn.c_proj.weight, residual=xm)
            return self.mlp(ops.norm(x), residual=x)
        if self.scalar_gate is not None:
            g = ops.linear(x[..., :self.gate_channels], self.scalar_gate.weight)
            x = (self.resid_lambda * (1.0 + g[..., 0:1])) * x + (self.x0_lambda * (1.0 + g[..., 1:2])) * x0
        elif self.x0_gate_s is not None:
            gate0 = 2.0 * torch.sigmoid(self.x0_gate_s * x.mean(dim=-1, keepdim=True))
            x = self.resid_lambda * x + self.x0_lambda * (gate0 * x0)
        else:
            x = self.resid_lambda * x + self.x0_lambda * x0
        x = x.to(x0.dtype)
        if self.block_nudge is not None and self.nudge_site == "resid":
            x = x + self.block_nudge.to(x.dtype) * x
        q_in = k_in = v_in = x
        if self.block_nudge is not None and self.nudge_site == "qk":
            q_in = k_in = x + self.block_nudge.to(x.dtype) * x
        if self.qk_shift_beta is not None:
            q_in = k_in = x + self.qk_shift_beta.to(x.dtype) * causal_shift_1(x)
        if self.local_conv is not None:
            x = x + self.local_conv(ops.norm(x))
            v_in = x if self.qk_shift_beta is None else v_in
            if self.qk_shift_beta is None:
                q_in = k_in = x
        if self.par_lambda_a is not None:
            h = ops.norm(x)
            attn_out = self.attn(h, h, h, ve, cos, sin, attn_mask, ve_bi, ve_tri)
            y = ops.linear(attn_out, self.attn.c_proj.weight)
            return x + self.par_lambda_a.to(x.dtype) * y + self.par_lambda_m.to(x.dtype) * self.mlp(h)
        hq = ops.norm(q_in)
        hk = hq if k_in is q_in else ops.norm(k_in)
        hv = hq if v_in is q_in else ops.norm(v_in)
        y = self.attn(hq, hk, hv, ve, cos, sin, attn_mask, ve_bi, ve_tri)
        x = ops.linear(y, self.attn.c_proj.weight, residual=x)
        if self.sandwich:
            return x + ops.norm(self.mlp(ops.norm(x)))
        return self.mlp(ops.norm(x), residual=x)


def _build_window_mask(T: int, window: int) -> torch.Tensor:
    i = torch.arange(T)[:, None]
    j = torch.arange(T)[None, :]
    keep = (j <= i) & (j > i - window)
    m = torch.zeros(T, T)
    m.masked_fill_(~keep, float("-inf"))
    return m


def doc_boundary_mask(idx: torch.Tensor, bos: int = 0) -> torch.Tensor:
    """Additive [B, 1, T, T] mask blocking attention across BOS-delimited documents."""
    doc = (idx == bos).cumsum(dim=1)
    same = doc[:, :, None] == doc[:, None, :]
    m = torch.zeros(same.shape, dtype=torch.float32, device=idx.device)
    m.masked_fill_(~same, float("-inf"))
    return m[:, None]


class GPT(nn.Module):
    def __init__(self, config: GPTConfig, rc: RunConfig | None = None):
        super().__init__()
        rc = rc or RunConfig()
        self.config = config
        self.rc = rc
        V = config.padded_vocab_size
        self.transformer = nn.ModuleDict({
            "wte": nn.Embedding(V, config.n_embd),
            "h": nn.ModuleList([Block(config, rc, i) for i in range(config.n_layer)]),
        })
        self.lm_head = Linear(config.n_embd, V)
        self.value_embeds = nn.ModuleDict({str(i): nn.Embedding(V, config.n_embd)
                                           for i in range(config.n_layer)
                                           if rc.ve and has_ve(i, config.n_layer)})
        self.ngram_rows = rc.ngram_ve_table_mult * V
        self.ngram_dim = rc.ngram_ve_dim if rc.ngram_ve_dim > 0 else config.n_embd
        tables = {}
        if rc.ngram_ve:
            self.ngram_mod = _largest_prime_below(self.ngram_rows) if self.ngram_rows < 5_000_000 else self.ngram_rows - 1
            dt = torch.bfloat16 if rc.ngram_ve_bf16 else torch.float32
            for i in sorted(_ngram_layers(rc.ngram_ve_layers, config.n_layer)):
                tables[f"b{i}"] = nn.Embedding(self.ngram_rows, self.ngram_dim,
                                               _weight=torch.zeros(self.ngram_rows, self.ngram_dim, dtype=dt))
                if rc.ngram_ve_trigram:
                    tables[f"t{i}"] = nn.Embedding(self.ngram_rows, self.ngram_dim,
                                                   _weight=torch.zeros(self.ngram_rows, self.ngram_dim, dtype=dt))
        self.ngram_embeds = nn.ModuleDict(tables)
        self.ngram_proj = nn.ModuleDict({k: Linear(self.ngram_dim, config.n_embd) for k in tables}
                                        if self.ngram_dim != config.n_embd else {})
        self.ngram_pad_id = V
        if rc.out_bigram:
            self.out_bigram = nn.Embedding(V, V, _weight=torch.zeros(
                V, V, dtype=torch.bfloat16 if rc.out_bigram_bf16 else torch.float32))
            self.out_bigram_gate = Linear(config.n_embd, 1)
            self.out_bigram_gate_bias = nn.Parameter(torch.full((1,), float(rc.out_bigram_gate_bias)))
        else:
            self.out_bigram = None
        self.out_pool_lambdas = (nn.Parameter(torch.zeros(min(rc.out_pool_layers, config.n_layer)))
                                 if rc.out_pool else None)
        # Engram-lite, built last among the table owners so it cannot shift their RNG draws
        self.engram_site = int(rc.engram_site) % config.n_layer if rc.engram else -1
        self.engram_share_keys: tuple[str, ...] = ()
        if rc.engram:
            share_dim = None
            if rc.engram_share_ngram_tables:
                self.engram_share_keys = tuple(k for k in self.ngram_embeds if int(k[1:]) <= self.engram_site)
                if not self.engram_share_keys:
                    raise ValueError("--engram-share-ngram-tables needs an n-gram table at or before the Engram site")
                share_dim = self.ngram_dim * len(self.engram_share_keys)
            self.engram = EngramLite(config, rc, V, share_dim)
        else:
            self.engram = None
        cos, sin = self._precompute_rotary_embeddings(config.sequence_len, config.head_dim)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)
        pattern = (rc.window_pattern * (config.n_layer // max(1, len(rc.window_pattern)) + 1))[:config.n_layer]
        self.layer_is_short = [c == "S" for c in pattern]
        if any(self.layer_is_short):
            short = max(1, int(config.sequence_len * rc.short_window_frac))
            self.register_buffer("mask_short", _build_window_mask(config.sequence_len, short), persistent=False)
        self.compute_dtype = torch.float32

    # ------------------------------------------------------------------ init
    def _precompute_rotary_embeddings(self, seq_len: int, head_dim: int, base: float | None = None):
        base = self.rc.rope_base if base is None else base
        freqs = torch.arange(0, head_dim, 2, dtype=torch.float32)
        inv_freq = 1.0 / (base ** (freqs / head_dim))
        t = torch.arange(seq_len, dtype=torch.float32)
        table = torch.outer(t, inv_freq)
        dt = torch.bfloat16 if self.compute_dtype_hint() == torch.bfloat16 else torch.float32
        return table.cos().to(dt)[None, :, None, :], table.sin().to(dt)[None, :, None, :]

    def compute_dtype_hint(self) -> torch.dtype:
        return getattr(self, "compute_dtype", torch.float32)

    def set_compute_dtype(self, dtype: torch.dtype) -> None:
        """bf16 on the GPU (the rotary tables follow), fp32 on the CPU oracle path."""
        self.compute_dtype = dtype
        cos, sin = self._precompute_rotary_embeddings(self.config.sequence_len, self.config.head_dim)
        self.cos = cos.to(self.cos.device)
        self.sin = sin.to(self.sin.device)

    @torch.no_grad()
    def init_weights(self) -> None:
        """Same distributions and RNG draw order as train.py:2957-3085 for the modules
        that exist (wte N(0, 0.8), lm_head N(0, 0.001), q/k/v U(+-s), attn c_proj
        U(+-0.1 s), c_fc U(+-0.4 s), mlp c_proj 0, lambdas 1 / 0.05, gates 0)."""
        rc = self.rc
        torch.nn.init.normal_(self.transformer.wte.weight, mean=0.0, std=rc.wte_init_std)
        torch.nn.init.normal_(self.lm_head.weight, mean=0.0, std=0.001)
        s = rc.init_scale * math.sqrt(3.0) * self.config.n_embd ** -0.5
        for block in self.transformer.h:
            torch.nn.init.uniform_(block.attn.c_q.weight, -s, s)
            torch.nn.init.uniform_(block.attn.c_k.weight, -s, s)
            torch.nn.init.uniform_(block.attn.c_v.weight, -s, s)
            if rc.attn_cproj_init_scale > 0.0:
                b = rc.attn_cproj_init_scale * s
                torch.nn.init.uniform_(block.attn.c_proj.weight, -b, b)
            else:
                torch.nn.init.zeros_(block.attn.c_proj.weight)
            torch.nn.init.uniform_(block.mlp.c_fc.weight, -0.4 * s, 0.4 * s)
            if block.mlp.c_gate is not None:
                torch.nn.init.uniform_(block.mlp.c_gate.weight, -0.4 * s, 0.4 * s)
            torch.nn.init.zeros_(block.mlp.c_proj.weight)
            block.resid_lambda.fill_(1.0)
            block.x0_lambda.fill_(0.05)
            if block.par_lambda_a is not None:
                block.par_lambda_a.fill_(1.0)
                block.par_lambda_m.fill_(1.0)
            if block.scalar_gate is not None:
                torch.nn.init.zeros_(block.scalar_gate.weight)
            for g in (block.attn.ve_gate, block.attn.ve_gate_bi, block.attn.ve_gate_tri):
                if g is not None:
                    torch.nn.init.zeros_(g.weight)
        for ve in self.value_embeds.values():
            torch.nn.init.uniform_(ve.weight, -s, s)
        for tbl in self.ngram_embeds.values():
            torch.nn.init.zeros_(tbl.weight)
        for proj in self.ngram_proj.values():
            torch.nn.init.uniform_(proj.weight, -s, s)
        if self.engram is not None:
            for tbl in self.engram.tables.values():
                torch.nn.init.zeros_(tbl.weight)
            for lin in (self.engram.w_k, self.engram.w_v, self.engram.w_q):
                if lin is not None:
                    torch.nn.init.uniform_(lin.weight, -s, s)
            if self.engram.conv is not None:
                torch.nn.init.zeros_(self.engram.conv.weight)
        if self.out_bigram is not None:
            torch.nn.init.zeros_(self.out_bigram.weight)
            torch.nn.init.zeros_(self.out_bigram_gate.weight)
        if self.out_pool_lambdas is not None:
            torch.nn.init.zeros_(self.out_pool_lambdas)
        for block in self.transformer.h:
            if block.attn.head_gate is not None:
                torch.nn.init.zeros_(block.attn.head_gate.weight)
        cos, sin = self._precompute_rotary_embeddings(self.config.sequence_len, self.config.head_dim)
        self.cos = cos.to(self.cos.device)
        self.sin = sin.to(self.sin.device)

    # ------------------------------------------------------------------ helpers
    def get_device(self) -> torch.device:
        return self.transformer.wte.weight.device

    def estimate_flops(self) -> int:
        """6 * (matmul params) + 12 * L * H * D * T per token (train.py:3191-3214)."""
        nparams = sum(p.numel() for p in self.parameters())
        non_matmul = self.transformer.wte.weight.numel() + 2 * self.config.n_layer
        non_matmul += sum(p.numel() for p in self.ngram_embeds.parameters())
        if self.engram is not None:
            non_matmul += sum(p.numel() for p in self.engram.tables.parameters())
        if self.out_bigram is not None:
            non_matmul += self.out_bigram.weight.numel()
        h, d, t = self.config.n_head, self.config.head_dim, self.config.sequence_len
        return 6 * (nparams - non_matmul) + self.config.n_layer * 12 * h * d * t

    def _ngram_hash_indices(self, idx: torch.Tensor) -> dict[str, torch.Tensor]:
        """Causal hashed n-gram ids: bigram (prev, cur), trigram (prev2, prev, cur);
        missing history = pad id one past the padded vocab (train.py:3087-3140)."""
        out = {}
        pad = self.ngram_pad_id
        cur = idx.long()
        prev = F.pad(cur[:, :-1], (1, 0), value=pad)
        prev2 = F.pad(cur[:, :-2], (2, 0), value=pad)
        if self.engram is not None:
            for key in self.engram.tables:
                head, order = int(key[1:key.index("o")]), int(key[key.index("o") + 1:])
                pr = engram_primes(head, order)
                hsh = (prev * pr[0]) ^ (cur * pr[1]) if order == 2 else (prev2 * pr[0]) ^ (prev * pr[1]) ^ (cur * pr[2])
                out[key] = hsh % self.engram.mod
        for key in self.ngram_embeds:
            layer = int(key[1:])
            p1, p2, p3 = _ngram_primes(layer)
            if key[0] == "b":
                hsh = (prev * p1) ^ (cur * p2)
            else:
                hsh = (prev2 * p1) ^ (prev * p2) ^ (cur * p3)
            out[key] = (hsh % self.ngram_mod)
        return out

    def _ngram_lookup(self, key: str, ids: torch.Tensor, dtype: torch.dtype, raw: dict | None = None,
                      idx: torch.Tensor | None = None) -> torch.Tensor:
        table = self.ngram_embeds[key].weight
        if idx is not None and table.is_cuda and not ops.oracle_active():
            # hash + gather in one kernel (the ids computed above are the same rows)
            order = 2 if key[0] == "b" else 3
            p = _ngram_primes(int(key[1:]))
            rows = ops.ngram_lookup(idx, table, order, p[:2] if order == 2 else p, self.ngram_mod,
                                    self.ngram_pad_id, dtype)
        else:
            rows = table[ids].to(dtype)
        if raw is not None:
            raw[key] = rows   # pre-projection rows, what a shared Engram memory reads
        if key in self.ngram_proj:
            rows = ops.linear(rows, self.ngram_proj[key].weight)
        return rows

    # ------------------------------------------------------------------ forward
    def enable_tp(self, tpc) -> None:
        """Run every block tensor-parallel over ``tpc`` (plain blocks only); the batch
        given to forward is then this rank's sequence shard of the group's micro-batch."""
        bad = [i for i, b in enumerate(self.transformer.h) if not b.plain]
        if bad or len(self.value_embeds) or len(self.ngram_embeds) or self.rc.doc_mask \
                or any(self.layer_is_short) or self.out_pool_lambdas is not None or self.out_bigram is not None or self.engram is not None:
            raise ValueError("tensor parallelism supports the plain block family only "
                             f"(non-plain layers: {bad}, or VE / n-gram / masks / pooling enabled)")
        self.tpc = tpc
        for i, b in enumerate(self.transformer.h):
            b._tpc = tpc
            b._layer_idx = i

    def enable_pp(self, ppc) -> None:
        """Run forward/backward as pipeline stage ``ppc.stage`` (plain-family blocks; VE,
        n-gram, Engram, pooling and masks are not staged)."""
        if len(self.value_embeds) or len(self.ngram_embeds) or self.engram is not None or self.rc.doc_mask \
                or any(self.layer_is_short) or self.out_pool_lambdas is not None or self.out_bigram is not None:
            raise ValueError("pipeline parallelism supports models without VE / n-gram / Engram / masks / pooling")
        self.ppc = ppc

    def disable_tp(self) -> None:
        """Back to whole-model blocks (every rank holds every weight whole), e.g. for an
        evaluation whose batches do not have the tensor-parallel row shape."""
        self.tpc = None
        for b in self.transformer.h:
            b._tpc = None

    def hidden(self, idx: torch.Tensor) -> torch.Tensor:
        """Final normed hidden states [B, T, C] (compute dtype)."""
        _b, t = idx.shape
        assert t <= self.config.sequence_len
        dt = self.compute_dtype
        cos, sin = self.cos[:, :t], self.sin[:, :t]
        x = ops.embed_norm(idx, self.transformer.wte.weight, dt)
        x0 = x
        doc_mask = doc_boundary_mask(idx) if self.rc.doc_mask else None
        ngram_idx = self._ngram_hash_indices(idx) if (len(self.ngram_embeds) or self.engram is not None) else None
        engram_raw = {} if (self.engram is not None and self.engram.share) else None
        pool_from = self.config.n_layer - self.out_pool_lambdas.numel() if self.out_pool_lambdas is not None else 1 << 30
        pool_buf = []
        for i, block in enumerate(self.transformer.h):
            ve = self.value_embeds[str(i)](idx.long()).to(dt) if str(i) in self.value_embeds else None
            ve_bi = ve_tri = None
            if ngram_idx is not None:
                if f"b{i}" in self.ngram_embeds:
                    ve_bi = self._ngram_lookup(f"b{i}", ngram_idx[f"b{i}"], dt, engram_raw, idx)
                if f"t{i}" in self.ngram_embeds:
                    ve_tri = self._ngram_lookup(f"t{i}", ngram_idx[f"t{i}"], dt, engram_raw, idx)
            if doc_mask is None and not self.layer_is_short[i]:
                attn_mask = None
            else:
                static = self.mask_short[:t, :t] if self.layer_is_short[i] else torch.zeros(t, t, device=idx.device)
                attn_mask = static.to(idx.device) + (doc_mask if doc_mask is not None else 0)
            x = block(x, x0, ve, cos, sin, attn_mask, ve_bi, ve_tri)
            if i == self.engram_site:
                if engram_raw is not None:
                    parts = [engram_raw[k] for k in self.engram_share_keys]
                    e_t = parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)
                else:
                    e_t = self.engram.gather(ngram_idx, dt)
                x = x + self.engram(x, e_t).to(x.dtype)
            if i >= pool_from:
                pool_buf.append(x)
        if self.out_pool_lambdas is not None:
            for k, h in enumerate(pool_buf):
                x = x + self.out_pool_lambdas[k].to(x.dtype) * h
        return ops.norm(x)

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None, loss_reduction: str = "mean",
                row_weight: torch.Tensor | None = None):
        x = self.hidden(idx)
        V = self.config.vocab_size
        S = self.rc.logit_softcap
        if self.out_bigram is not None:
            logits = F.linear(x, self.lm_head.weight.to(x.dtype))[..., :V].float()
            g = torch.sigmoid(ops.linear(x, self.out_bigram_gate.weight) + self.out_bigram_gate_bias.to(x.dtype))
            row = self.out_bigram.weight[idx.long()][..., :V]
            logits = logits + (g * row.to(g.dtype)).float()
            if targets is None:
                return S * torch.tanh(logits / S)
            return ops.ref.softcap_cross_entropy(logits, targets, S, loss_reduction,
                                                 None if row_weight is None else row_weight.reshape(-1))
        if targets is None:
            return ops.softcap_logits(x, self.lm_head.weight, S, V)
        return ops.lm_head_softcap_ce(x, self.lm_head.weight, targets, S, V, loss_reduction, row_weight)

    def model_config_dict(self) -> dict:
        return asdict(self.config)
