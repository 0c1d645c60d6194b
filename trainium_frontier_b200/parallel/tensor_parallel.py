"""Tensor parallelism (Megatron column/row split with sequence-parallel activations).

A tensor-parallel group of ``tp`` ranks shares one micro-batch.  Each rank owns whole
sequences of it for everything outside the attention/MLP matmuls (embedding, norms,
residual stream, lm_head + loss): its "sequence shard" of ``rows_per_rank`` token rows.
Inside a block each rank owns a slice of the heads and of the MLP hidden units:

    h_sp  --all-gather-->  [M, C]  @ W_qkv[heads_t]^T   -> attention on heads_t (all rows)
    y[M, heads_t] @ W_proj[:, heads_t]^T  --reduce-scatter-->  + x_sp   (own rows)
    hn_sp --all-gather-->  [M, C]  @ W_fc[hidden_t]^T -> relu^2
    u[M, hidden_t] @ W_mproj[:, hidden_t]^T --reduce-scatter--> + x1_sp

On CUDA the all-gather and the reduce-scatter are fused into the tcgen05 GEMM kernel
(``gemm_tp``: MODE_AG pulls the peers' rows over NVLink into a symmetric gather buffer
while the MMAs start on the local rows; MODE_RS stores the peers' partial tiles straight
into their receive buffers and sums the arriving partials in the epilogue).  On the
CPU the same block runs on ``all_gather`` / ``all_reduce`` (gloo) so the sharding and
gradient math can be tested without a GPU.

Parameters stay replicated and whole on every rank (the checkpoint layout is the
single-device one; nothing to consolidate).  A rank only computes with, and only writes
gradients into, its own slices; the other slices' gradients stay zero.  Each rank
back-propagates the mean loss of its own rows, and the data-parallel engine averages
the flat gradient buffer over ALL ranks: for a sharded matrix the TP group's backward
already sums both ranks' loss gradients (2 L per group), for a replicated parameter
each rank holds its own rows' part, so in both cases the all-rank mean is the mean over
data-parallel groups of the group-mean loss gradient.  Muon then sees whole matrices
(distributed Muon assigns each whole matrix to one owner rank).

The reference has no tensor parallelism (it trains pure data parallel,
``train.py:4383-4528``); this is the d26 / seq 4096 TP=2 x DP=4 configuration.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd import Function

BF16 = torch.bfloat16
MODE_AG, MODE_RS = 1, 2
EPI_BF16, EPI_RELU2, EPI_RELU2_BWD = 0, 1, 2


def tp_split(n: int, tp: int, t: int, unit: int) -> tuple[int, int]:
    """(start, count) of rank t's share of n elements cut into `unit`-sized pieces."""
    assert n % unit == 0, (n, unit)
    units = n // unit
    base, rem = divmod(units, tp)
    cnt = base + (1 if t < rem else 0)
    start = t * base + min(t, rem)
    return start * unit, cnt * unit


class TPContext:
    """Process groups, symmetric buffers and call epochs of one tensor-parallel group."""

    def __init__(self, tp: int, device: torch.device, rows_per_rank: int, width: int, n_slots: int):
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        if self.world % tp:
            raise ValueError(f"world {self.world} is not a multiple of tp={tp}")
        self.tp, self.dp = tp, self.world // tp
        self.tp_rank, self.dp_rank = self.rank % tp, self.rank // tp
        self.device = device
        self.Mr, self.M, self.C = rows_per_rank, rows_per_rank * tp, width
        self.pg = None
        for d in range(self.dp):
            g = dist.new_group(list(range(d * tp, (d + 1) * tp)))
            if d == self.dp_rank:
                self.pg = g
        self.own = slice(self.tp_rank * rows_per_rank, (self.tp_rank + 1) * rows_per_rank)
        self.n_slots = n_slots
        self.epoch = 0
        self.rs_calls = 0
        self.bwd_calls = 0
        self.weights_version = 0
        self.cuda = device.type == "cuda"
        if self.cuda:
            self._init_symm()
        else:
            self.slots = [torch.zeros(self.M, width, device=device) for _ in range(n_slots + 2)]

    # ------------------------------------------------------------------ CUDA buffers
    def _init_symm(self) -> None:
        import torch.distributed._symmetric_memory as symm_mem
        from ..ops._ext import C, err_word
        if self.Mr % 128:
            raise ValueError(f"rows per rank ({self.Mr}) must be a multiple of 128")
        if self.C % 8:
            raise ValueError("model width must be a multiple of 8")
        tp, dev = self.tp, self.device
        self.C_ = C
        self.err = err_word(dev)
        slot_elems = self.M * self.C
        self.gpool = symm_mem.empty((self.n_slots + 2) * slot_elems, dtype=BF16, device=dev)
        h = symm_mem.rendezvous(self.gpool, self.pg)
        self._h = [h]
        base = self.gpool.data_ptr()
        off = base - int(h.buffer_ptrs[self.tp_rank])
        self.g_peers = [int(p) + off for p in h.buffer_ptrs]
        self.slot_bytes = slot_elems * 2
        self.slots = [self.gpool[i * slot_elems:(i + 1) * slot_elems].view(self.M, self.C)
                      for i in range(self.n_slots + 2)]
        # ready pads [tp] + RS flags 2 x [tp][tiles][8] (lane quarter x column half) in one
        # symmetric int32 buffer
        tiles_n = (self.C + 127) // 128
        self.rs_tiles = (self.Mr // 128) * tiles_n
        flag_words = tp + 2 * tp * self.rs_tiles * 8
        self.flags = symm_mem.empty(flag_words, dtype=torch.int32, device=dev)
        self.flags.zero_()
        fh = symm_mem.rendezvous(self.flags, self.pg)
        self._h.append(fh)
        foff = self.flags.data_ptr() - int(fh.buffer_ptrs[self.tp_rank])
        fpeers = [int(p) + foff for p in fh.buffer_ptrs]
        self.ready_peers = fpeers
        self.rsflag_peers = [[p + 4 * (tp + par * tp * self.rs_tiles * 8) for p in fpeers] for par in range(2)]
        recv_elems = tp * self.Mr * self.C
        self.recv = symm_mem.empty(2 * recv_elems, dtype=BF16, device=dev)
        rh = symm_mem.rendezvous(self.recv, self.pg)
        self._h.append(rh)
        roff = self.recv.data_ptr() - int(rh.buffer_ptrs[self.tp_rank])
        self.recv_peers = [[int(p) + roff + 2 * par * recv_elems for p in rh.buffer_ptrs] for par in range(2)]
        self.sched = torch.zeros(4, dtype=torch.int32, device=dev)
        self.claim = torch.zeros(max(1, (tp - 1) * self.Mr // 128), dtype=torch.int32, device=dev)
        self.done = torch.zeros(self.M // 128, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.pg)

    def slot(self, i: int) -> torch.Tensor:
        return self.slots[i]

    def bwd_slot(self) -> int:
        self.bwd_calls += 1
        return self.n_slots + (self.bwd_calls & 1)

    # ------------------------------------------------------------------ primitives
    def put_rows(self, slot: int, x_sp: torch.Tensor) -> torch.Tensor:
        """Write this rank's rows of a gather slot; returns the slot [M, C]."""
        s = self.slots[slot]
        s[self.own].copy_(x_sp.reshape(self.Mr, self.C))
        return s

    def ag_gemm(self, slot: int, w: torch.Tensor, b_mn: bool, epi: int = EPI_BF16, D2=None, R=None,
                tau: float = 0.0) -> torch.Tensor:
        """out[M, N] = gather(slot) @ op(w); op(w) = w^T ([N, C]) or w ([C, N] if b_mn).
        The slot's own rows must already be written (put_rows)."""
        N = w.shape[1] if b_mn else w.shape[0]
        out = torch.empty(self.M, N, dtype=BF16 if self.cuda else torch.float32, device=self.device)
        if not self.cuda:
            full = self.slots[slot]
            parts = [torch.empty_like(full[self.own]) for _ in range(self.tp)]
            dist.all_gather(parts, full[self.own].contiguous(), group=self.pg)
            full.copy_(torch.cat(parts, 0))
            z = full @ (w if b_mn else w.t())
            if epi == EPI_RELU2:
                D2.copy_(z)
                out.copy_(torch.relu(z - tau).square())
            elif epi == EPI_RELU2_BWD:
                out.copy_(z * 2 * torch.relu(R - tau))
            else:
                out.copy_(z)
            return out
        from ..ops.gemm import _bn
        self.epoch += 1
        self.C_().gemm_tp(MODE_AG, self.slots[slot], w, b_mn, self.M, N, self.C, out, epi, R, D2, float(tau), 1.0,
                          self.tp_rank, self.tp, self.Mr, self.epoch, [p + slot * self.slot_bytes for p in self.g_peers],
                          self.ready_peers, self.claim, self.done, [], [], self.sched, _bn(N), self.err)
        return out

    def rs_gemm(self, a: torch.Tensor, w: torch.Tensor, b_mn: bool, residual: torch.Tensor | None = None) -> torch.Tensor:
        """out_sp[Mr, C] = (a @ op(w))[own rows summed over the group] (+ residual);
        a [M, K], op(w) = w^T ([C, K]) or w ([K, C] if b_mn)."""
        K = a.shape[1]
        out = torch.empty(self.Mr, self.C, dtype=BF16 if self.cuda else torch.float32, device=self.device)
        if not self.cuda:
            z = a @ (w if b_mn else w.t())
            dist.all_reduce(z, group=self.pg)
            out.copy_(z[self.own])
            if residual is not None:
                out += residual.reshape(self.Mr, self.C)
            return out
        from ..ops.gemm import _bn
        self.epoch += 1
        par = self.rs_calls & 1
        self.rs_calls += 1
        R = residual.reshape(self.Mr, self.C) if residual is not None else None
        self.C_().gemm_tp(MODE_RS, a, w, b_mn, self.M, self.C, K, out, EPI_BF16, R, None, 0.0, 1.0,
                          self.tp_rank, self.tp, self.Mr, self.epoch, [], [], None, None,
                          self.recv_peers[par], self.rsflag_peers[par], self.sched, _bn(self.C), self.err)
        return out

    def close(self) -> None:
        if self.cuda:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pg)
            self._h = []


# --------------------------------------------------------------------------- autograd
def _dw(dy: torch.Tensor, x: torch.Tensor, g: torch.Tensor) -> None:
    """g[N, K] += dy[M, N]^T x[M, K] (fp32 gradient view)."""
    if dy.is_cuda:
        from ..ops.gemm import linear_dw
        linear_dw(dy, x, g)
    else:
        g += dy.t().float() @ x.float()


class TPColumnFn(Function):
    """out[M, N_t] = gather(x_sp) @ W_t^T, W_t the rows of this rank (qkv: [q_t; k_t; v_t])."""

    @staticmethod
    def forward(ctx, x_sp, w, grads, tpc, slot):
        tpc.put_rows(slot, x_sp)
        out = tpc.ag_gemm(slot, w, False)
        ctx.w, ctx.grads, ctx.tpc, ctx.slot = w, grads, tpc, slot
        ctx.shape = x_sp.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        tpc, w = ctx.tpc, ctx.w
        dout = dout.reshape(tpc.M, -1)
        dx = tpc.rs_gemm(dout, w, True)
        x_full = tpc.slot(ctx.slot)
        c0 = 0
        for g in ctx.grads:
            n = g.shape[0]
            _dw(dout[:, c0:c0 + n], x_full, g)
            c0 += n
        return dx.view(ctx.shape), None, None, None, None


class TPRowFn(Function):
    """out_sp = reduce_scatter(y @ W_t^T) + residual_sp, W_t = W[:, cols_t] ([C, N_t])."""

    @staticmethod
    def forward(ctx, y, w, grad, residual, tpc):
        y2 = y.reshape(tpc.M, -1)
        out = tpc.rs_gemm(y2, w, False, residual)
        ctx.save_for_backward(y2)
        ctx.w, ctx.grad, ctx.tpc = w, grad, tpc
        ctx.yshape = y.shape
        return out.view(residual.shape)

    @staticmethod
    def backward(ctx, dout):
        (y2,) = ctx.saved_tensors
        tpc = ctx.tpc
        slot = tpc.bwd_slot()
        tpc.put_rows(slot, dout)
        dy = tpc.ag_gemm(slot, ctx.w, True)          # [M, N_t] = dout_full @ W_t
        _dw(tpc.slot(slot), y2, ctx.grad)           # dW_t[C, N_t] += dout_full^T y
        return dy.view(ctx.yshape), None, None, dout, None


class TPMLPFn(Function):
    """out_sp = reduce_scatter(relu(gather(x_sp) W_fc_t^T - tau)^2 W_mp_t^T) + residual_sp."""

    @staticmethod
    def forward(ctx, x_sp, w_fc, g_fc, w_mp, g_mp, residual, tpc, slot, tau):
        tpc.put_rows(slot, x_sp)
        Ft = w_fc.shape[0]
        h = torch.empty(tpc.M, Ft, dtype=BF16 if tpc.cuda else torch.float32, device=x_sp.device)
        u = tpc.ag_gemm(slot, w_fc, False, EPI_RELU2, D2=h, tau=tau)
        out = tpc.rs_gemm(u, w_mp, False, residual)
        ctx.save_for_backward(u, h)
        ctx.w = (w_fc, g_fc, w_mp, g_mp)
        ctx.tpc, ctx.slot, ctx.tau = tpc, slot, tau
        return out.view(residual.shape)

    @staticmethod
    def backward(ctx, dout):
        u, h = ctx.saved_tensors
        w_fc, g_fc, w_mp, g_mp = ctx.w
        tpc = ctx.tpc
        slot = tpc.bwd_slot()
        tpc.put_rows(slot, dout)
        dh = tpc.ag_gemm(slot, w_mp, True, EPI_RELU2_BWD, R=h, tau=ctx.tau)   # [M, F_t]
        _dw(tpc.slot(slot), u, g_mp)                                           # [C, F_t]
        dx = tpc.rs_gemm(dh, w_fc, True)                                       # [Mr, C]
        _dw(dh, tpc.slot(ctx.slot), g_fc)                                      # [F_t, C]
        return dx.view(dout.shape), None, None, None, None, dout, None, None, None


# --------------------------------------------------------------------------- block
class TPShards:
    """This rank's weight slices of one block (bf16 compute views + fp32 gradient views)."""

    def __init__(self, blk, tpc: TPContext):
        a, m = blk.attn, blk.mlp
        D = a.head_dim
        self.q0, self.nq = tp_split(a.n_head * D, tpc.tp, tpc.tp_rank, D)
        self.heads = self.nq // D
        F = m.c_fc.weight.shape[0]
        self.f0, self.nf = tp_split(F, tpc.tp, tpc.tp_rank, 128 if F % (128 * tpc.tp) == 0 else 8)
        self.blk, self.tpc = blk, tpc
        self.version = -1
        self.wqkv = None

    def _w(self, p):
        from ..ops.fused import w16
        return w16(p) if self.tpc.cuda else p.detach()

    def _g(self, p):
        from ..ops.fused import grad_buf
        return grad_buf(p)

    def qkv(self):
        a = self.blk.attn
        sl = slice(self.q0, self.q0 + self.nq)
        if self.wqkv is None or self.version != self.tpc.weights_version or not self.tpc.cuda:
            self.wqkv = torch.cat([self._w(a.c_q.weight)[sl], self._w(a.c_k.weight)[sl], self._w(a.c_v.weight)[sl]], 0)
            self.version = self.tpc.weights_version
        return self.wqkv, [self._g(a.c_q.weight)[sl], self._g(a.c_k.weight)[sl], self._g(a.c_v.weight)[sl]]

    def proj(self):
        p = self.blk.attn.c_proj.weight
        sl = slice(self.q0, self.q0 + self.nq)
        return self._w(p)[:, sl], self._g(p)[:, sl]

    def mlp(self):
        m = self.blk.mlp
        sl = slice(self.f0, self.f0 + self.nf)
        return (self._w(m.c_fc.weight)[sl], self._g(m.c_fc.weight)[sl],
                self._w(m.c_proj.weight)[:, sl], self._g(m.c_proj.weight)[:, sl])


def block_forward_tp(blk, x, x0, cos, sin, tpc: TPContext, layer_idx: int):
    """Tensor-parallel forward of a plain block on this rank's sequence shard x [Bl, T, C]."""
    from .. import ops
    sh = getattr(blk, "_tp_shards", None)
    if sh is None or sh.tpc is not tpc:
        sh = blk._tp_shards = TPShards(blk, tpc)
    a = blk.attn
    Bl, T, Cw = x.shape
    Bg = Bl * tpc.tp
    D = a.head_dim
    xm, h = ops.mix_norm(x, x0, blk.resid_lambda, blk.x0_lambda)
    wqkv, gqkv = sh.qkv()
    qkv = TPColumnFn.apply(h, wqkv, gqkv, tpc, 2 * layer_idx)
    y = ops.attention_qkv(qkv.view(Bg, T, 3 * sh.nq), cos, sin, sh.heads, D, a.attn_scale)
    wp, gp = sh.proj()
    x1 = TPRowFn.apply(y, wp, gp, xm, tpc)
    wf, gf, wm, gm = sh.mlp()
    return TPMLPFn.apply(ops.norm(x1), wf, gf, wm, gm, x1, tpc, 2 * layer_idx + 1, blk.mlp.tau)
