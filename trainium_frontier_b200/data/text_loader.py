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
