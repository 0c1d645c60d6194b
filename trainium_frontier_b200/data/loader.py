"""Training and evaluation loaders over the synthetic corpus.

``make_dataloader`` keeps the reference's contract (``prepare.py:456-518``): an
infinite generator of ``(inputs int32 [B, T], targets int64 [B, T], {"epoch": e})``
with BOS-aligned best-fit packing, pinned host staging and a non-blocking H2D copy.

``PackedRowLoader`` is the engine's own form: it moves ONE int32 ``[B, T+1]`` row
block per micro-step (4 bytes/token instead of the reference's 12) from pinned host
memory on a side stream, double-buffered, and the kernels read inputs/targets as
the two shifted views of that block.

``make_eval_dataloader`` mirrors ``prepare.py:521-585``: a finite stream chunked into
rows with stride ``seq_len`` (no packing), targets -1 past the valid tail, and a final
batch padded with BOS / -1.
"""
from __future__ import annotations

import torch

from ..runtime import get_dist_info
from . import synthetic as syn


def _packer(split: str, rank: int, seed: int | None = None, vocab: int = 8192):
    base = seed if seed is not None else (syn.TRAIN_SEED if split == "train" else syn.VAL_SEED)
    return syn.native().BestFitPacker(vocab, syn.ZIPF_S, syn.MEAN_DOC_LEN,
                                      syn.rank_seed(base, rank), syn.BOS_ID, 512)


class EpochPacker:
    """The train split as a corpus of finite epochs (``epoch_rows`` packed rows per rank).

    With ``epoch_rows == 0`` the stream is endless (one epoch).  Otherwise epoch 1 is the
    split's seeded order, and when it is used up the next epoch begins: without shuffling
    it replays epoch 1 exactly (the same documents in the same order, as a finite corpus
    read twice would), with ``shuffle`` epoch ``e`` is a fresh order seeded by
    ``shuffle_seed + e`` -- the reference's requeue packer reshuffles its row groups
    from epoch 2 on in the same way (``train.py:106-196``, ``--epoch-shuffle``)."""

    def __init__(self, split: str, rank: int, seed: int | None = None, vocab: int = 8192,
                 epoch_rows: int = 0, shuffle: bool = False, shuffle_seed: int = 1234):
        self.split, self.rank, self.seed, self.vocab = split, rank, seed, vocab
        self.epoch_rows, self.shuffle, self.shuffle_seed = int(epoch_rows), bool(shuffle), int(shuffle_seed)
        self.epoch = 1
        self.rows_left = self.epoch_rows
        self.packer = _packer(split, rank, seed, vocab)

    def _start_next_epoch(self) -> None:
        self.epoch += 1
        seed = self.seed
        if self.shuffle:
            base = seed if seed is not None else (syn.TRAIN_SEED if self.split == "train" else syn.VAL_SEED)
            seed = base + self.shuffle_seed + self.epoch
        self.packer = _packer(self.split, self.rank, seed, self.vocab)
        self.rows_left = self.epoch_rows

    def fill(self, rows: torch.Tensor) -> None:
        if self.epoch_rows <= 0:
            self.packer.fill(rows)
            return
        done = 0
        while done < rows.shape[0]:
            if self.rows_left == 0:
                self._start_next_epoch()
            n = min(self.rows_left, rows.shape[0] - done)
            self.packer.fill(rows[done:done + n])
            done += n
            self.rows_left -= n


def make_dataloader(tokenizer, batch_size: int, seq_len: int, split: str,
                    device: torch.device | str, seed: int | None = None, epoch_tokens: int = 0,
                    epoch_shuffle: bool = False, epoch_shuffle_seed: int = 1234, **_unused):
    """BOS-aligned best-fit packed loader with the reference's yield contract; the third
    item's ``epoch`` counts epochs of ``epoch_tokens`` tokens per rank (see ``EpochPacker``)."""
    assert batch_size > 0 and seq_len > 1
    _ddp, rank, _lr, _ws = get_dist_info()
    vocab = tokenizer.get_vocab_size() if tokenizer is not None else 8192
    packer = EpochPacker(split, rank, seed, vocab, epoch_rows=_epoch_rows(epoch_tokens, seq_len),
                         shuffle=epoch_shuffle, shuffle_seed=epoch_shuffle_seed)
    dev = torch.device(device)
    pin = dev.type == "cuda"
    rows = torch.empty((batch_size, seq_len + 1), dtype=torch.int32)
    cpu_inputs = torch.empty((batch_size, seq_len), dtype=torch.int32, pin_memory=pin)
    cpu_targets = torch.empty((batch_size, seq_len), dtype=torch.long, pin_memory=pin)
    inputs = torch.empty((batch_size, seq_len), dtype=torch.int32, device=dev)
    targets = torch.empty((batch_size, seq_len), dtype=torch.long, device=dev)
    while True:
        packer.fill(rows)
        cpu_inputs.copy_(rows[:, :-1])
        cpu_targets.copy_(rows[:, 1:])
        inputs.copy_(cpu_inputs, non_blocking=pin)
        targets.copy_(cpu_targets, non_blocking=pin)
        yield inputs, targets, {"epoch": packer.epoch}


def _epoch_rows(epoch_tokens: int, seq_len: int) -> int:
    return 0 if epoch_tokens <= 0 else max(1, epoch_tokens // (seq_len + 1))


class PackedRowLoader:
    """Double-buffered pinned-host -> device loader of packed ``[B, T+1]`` int32 rows.

    ``next()`` returns a device tensor; the copy of the following block is already in
    flight on a dedicated stream, and the consumer stream waits on its event, so the
    H2D transfer overlaps compute.  ``h2d_bytes_per_batch`` reports exactly what crosses
    PCIe per micro-step.
    """

    def __init__(self, batch_size: int, seq_len: int, device: torch.device, split: str = "train",
                 seed: int | None = None, rank: int | None = None, vocab: int = 8192, depth: int = 2,
                 epoch_tokens: int = 0, epoch_shuffle: bool = False, epoch_shuffle_seed: int = 1234,
                 packer=None):
        if rank is None:
            rank = get_dist_info()[1]
        self.B, self.T = batch_size, seq_len
        self.device = torch.device(device)
        # any object with fill(host int32 [B, T+1]) can stand in for the synthetic stream
        # (data.text_loader.TextPacker for text files)
        self.packer = packer if packer is not None else EpochPacker(
            split, rank, seed, vocab, epoch_rows=_epoch_rows(epoch_tokens, seq_len), shuffle=epoch_shuffle,
            shuffle_seed=epoch_shuffle_seed)
        cuda = self.device.type == "cuda"
        self.depth = depth
        self.host = [torch.empty((batch_size, seq_len + 1), dtype=torch.int32, pin_memory=cuda)
                     for _ in range(depth)]
        self.dev = [torch.empty((batch_size, seq_len + 1), dtype=torch.int32, device=self.device)
                    for _ in range(depth)]
        self.stream = torch.cuda.Stream(self.device) if cuda else None
        self.events = [torch.cuda.Event() if cuda else None for _ in range(depth)]
        self.free = [torch.cuda.Event() if cuda else None for _ in range(depth)]
        self.i = 0
        self._issue(0)

    @property
    def h2d_bytes_per_batch(self) -> int:
        return self.B * (self.T + 1) * 4

    def _issue(self, slot: int) -> None:
        if self.stream is not None:
            # the host buffer may still be read by an earlier async copy
            self.free[slot].synchronize()
        self.packer.fill(self.host[slot])
        if self.stream is None:
            self.dev[slot].copy_(self.host[slot])
            return
        with torch.cuda.stream(self.stream):
            self.dev[slot].copy_(self.host[slot], non_blocking=True)
            self.events[slot].record(self.stream)
            self.free[slot].record(self.stream)

    def next(self) -> torch.Tensor:
        slot = self.i % self.depth
        nxt = (self.i + 1) % self.depth
        if self.stream is not None:
            torch.cuda.current_stream(self.device).wait_event(self.events[slot])
        out = self.dev[slot]
        self.i += 1
        # The consumer must be done with dev[nxt] before it is overwritten: record the
        # consumer stream position and make the copy stream wait on it.
        if self.stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.stream.wait_event(ev)
        self._issue(nxt)
        return out

    def __iter__(self):
        return self

    @property
    def epoch(self) -> int:
        """Epoch of the most recently packed rows (one block ahead of ``next()``)."""
        return self.packer.epoch

    def __next__(self):
        rows = self.next()
        return rows[:, :-1], rows[:, 1:], {"epoch": self.packer.epoch}


def _to_dev(bx, by, dev):
    """Rows -> (x int32, y int64) on `dev`; on CUDA through pinned host memory."""
    x = torch.tensor(bx, dtype=torch.int32)
    y = torch.tensor(by, dtype=torch.long)
    if dev.type == "cuda":
        x, y = x.pin_memory().to(dev, non_blocking=True), y.pin_memory().to(dev, non_blocking=True)
    elif dev != x.device:
        x, y = x.to(dev), y.to(dev)
    return x, y, {"documents": 0}


def make_eval_dataloader(tokenizer, batch_size: int, seq_len: int, split: str,
                         device: torch.device | str, max_stream_tokens: int = 1 << 21,
                         seed: int | None = None, **_unused):
    """Finite eval loader: a per-rank token stream chunked into rows of stride ``seq_len``
    (reference ``prepare.py:521-585``): the synthetic held-out stream, or, when the
    tokenizer carries ``eval_documents(rank, world)`` (an iterable of held-out text), those
    documents tokenized with BOS first."""
    assert batch_size > 0 and seq_len > 1
    _ddp, rank, _lr, world = get_dist_info()
    vocab = tokenizer.get_vocab_size() if tokenizer is not None else 8192
    n_local = max(seq_len + 1, (max_stream_tokens + world - 1) // world)
    docs_fn = getattr(tokenizer, "eval_documents", None)
    if docs_fn is not None:
        # held-out text: this rank's documents, BOS first, back to back
        bos = tokenizer.get_bos_token_id()
        stream = []
        chunk = []
        for s_ in docs_fn(rank, world):
            chunk.append(s_)
            if len(chunk) == 128:
                for ids in tokenizer.encode(chunk, prepend=bos):
                    stream.extend(ids)
                chunk = []
                if len(stream) >= n_local:
                    break
        if chunk and len(stream) < n_local:
            for ids in tokenizer.encode(chunk, prepend=bos):
                stream.extend(ids)
        stream = stream[:n_local]
    else:
        bos = syn.BOS_ID
        packer = _packer(split, rank, seed, vocab)
        stream_t = torch.empty(n_local, dtype=torch.int32)
        packer.fill_stream(stream_t)
        stream = stream_t.tolist()
    dev = torch.device(device)
    bx: list[list[int]] = []
    by: list[list[int]] = []
    pos = 0
    while pos + seq_len + 1 <= len(stream):
        row = stream[pos:pos + seq_len + 1]
        bx.append(row[:-1])
        by.append(row[1:])
        pos += seq_len
        if len(bx) == batch_size:
            yield _to_dev(bx, by, dev)
            bx, by = [], []
    tail = stream[pos:]
    if len(tail) > 1:
        valid = len(tail) - 1
        row = tail + [bos] * (seq_len + 1 - len(tail))
        bx.append(row[:-1])
        by.append(row[1:valid + 1] + [-1] * (seq_len - valid))
    if bx:
        while len(bx) < batch_size:
            bx.append([bos] * seq_len)
            by.append([-1] * seq_len)
        yield _to_dev(bx, by, dev)
