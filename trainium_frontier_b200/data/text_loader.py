"""Training rows from real text: documents tokenized with a ``Tokenizer`` (BOS first) and
packed BOS-aligned best-fit by the native ``DocPacker`` (the packing of the synthetic
path, fed by the caller instead of a generator).

    docs = parquet_documents(["shard_00000.parquet", ...])            # or any iterable of str
    for x, y in text_dataloader(tokenizer, docs, batch_size=32, seq_len=2048, device="cuda"):
        ...

Each batch is ``(inputs int32 [B, T], targets int64 [B, T])`` from rows of T + 1 tokens,
copied to ``device`` from pinned host memory; it ends when the documents run out (the last
incomplete row is dropped).  ``rank`` / ``world`` stride the documents over data-parallel
ranks (or let ``parquet_documents`` stride row groups instead; use one of the two).
Reference counterpart: ``make_dataloader`` (``prepare.py:456-518``) over its parquet row
groups (``prepare.py:423-444``).
"""
from __future__ import annotations

from typing import Iterable, Iterator

import torch

BUFFER_MIN = 512    # documents held for the best-fit search (the reference's buffer)
ENCODE_CHUNK = 128  # documents tokenized per batch call


def _native():
    from .. import _native
    return _native


def parquet_documents(paths, column: str = "text", rank: int = 0, world: int = 1) -> Iterator[str]:
    """The ``column`` strings of parquet files, row group by row group; rank ``rank`` of
    ``world`` takes every ``world``-th row group (the reference's rank striding)."""
    import pyarrow.parquet as pq
    g = 0
    for path in paths:
        f = pq.ParquetFile(path)
        for i in range(f.num_row_groups):
            if g % world == rank:
                for s in f.read_row_group(i, columns=[column]).column(column).to_pylist():
                    if s:
                        yield s
            g += 1


def text_dataloader(tokenizer, documents: Iterable[str], batch_size: int, seq_len: int, device="cpu",
                    rank: int = 0, world: int = 1, buffer_min: int = BUFFER_MIN,
                    num_threads: int = 4) -> Iterator[tuple[torch.Tensor, torch.Tensor]]:
    dev = torch.device(device)
    bos = tokenizer.get_bos_token_id()
    packer = _native().DocPacker(buffer_min)
    docs = iter(documents)
    exhausted = False
    # the buffer is topped up to buffer_min + margin before each fill: a row of T + 1 tokens
    # takes at most (T + 1) / 2 documents (every document is BOS + at least one token), so
    # a row never runs the buffer dry while documents remain
    margin = (seq_len + 1) // 2 + 1
    k = 0

    def refill() -> bool:
        nonlocal exhausted, k
        while not exhausted and packer.buffered() < buffer_min + margin:
            chunk = []
            while len(chunk) < ENCODE_CHUNK:
                try:
                    s = next(docs)
                except StopIteration:
                    exhausted = True
                    break
                if k % world == rank:
                    chunk.append(s)
                k += 1
            if chunk:
                for ids in tokenizer.encode(chunk, prepend=bos, num_threads=num_threads):
                    packer.push(torch.tensor(ids, dtype=torch.int64))
        return not exhausted

    pin = dev.type == "cuda"
    while True:
        rows = torch.empty(batch_size, seq_len + 1, dtype=torch.int32, pin_memory=pin)
        r = 0
        while r < batch_size:
            refill()
            got = packer.fill(rows, r, exhausted)
            r += got
            if got == 0 and (exhausted or packer.buffered() == 0):
                return
        x = rows[:, :-1].to(dev, non_blocking=pin)
        y = rows[:, 1:].to(dev, dtype=torch.int64, non_blocking=pin)
        yield x, y


class TextPacker:
    """Endless packed rows from text files for the trainer: ``fill(rows)`` fills a host
    ``[B, T+1]`` int32 tensor (the interface of the synthetic packers, so
    ``PackedRowLoader`` double-buffers it the same way), starting the next epoch over the
    files when the documents run out.  Rank ``rank`` of ``world`` reads every
    ``world``-th parquet row group."""

    def __init__(self, tokenizer, paths, rank: int = 0, world: int = 1, column: str = "text",
                 buffer_min: int = BUFFER_MIN, num_threads: int = 4):
        self.tok, self.paths, self.rank, self.world = tokenizer, list(paths), rank, world
        self.column, self.buffer_min, self.num_threads = column, buffer_min, num_threads
        if not self.paths:
            raise ValueError("no text data files")
        self.packer = _native().DocPacker(buffer_min)
        self.epoch = 0
        self._docs = parquet_documents(self.paths, column, rank, world)

    def _top_up(self, want: int) -> None:
        bos = self.tok.get_bos_token_id()
        fresh_epoch = False
        while self.packer.buffered() < want:
            chunk = []
            for s in self._docs:
                chunk.append(s)
                if len(chunk) == ENCODE_CHUNK:
                    break
            if not chunk:
                if fresh_epoch:
                    raise ValueError("the text data holds too few documents to fill the packing buffer")
                self.epoch += 1
                fresh_epoch = True
                self._docs = parquet_documents(self.paths, self.column, self.rank, self.world)
                continue
            fresh_epoch = False
            for ids in self.tok.encode(chunk, prepend=bos, num_threads=self.num_threads):
                self.packer.push(torch.tensor(ids, dtype=torch.int64))

    def fill(self, rows: torch.Tensor) -> None:
        want = self.buffer_min + rows.shape[1] // 2 + 1
        r = 0
        while r < rows.shape[0]:
            self._top_up(want)
            r += self.packer.fill(rows, r, False)
