"""Seeded synthetic corpus: Zipf token documents and a per-token byte-length table.

No dataset or tokenizer can be fetched on the target machines, so every run uses a
deterministic synthetic stream with the statistics the benchmark configuration names:
token ids from Zipf(s=1.1) over [1, vocab) with BOS = 0 starting each document, and
document lengths geometric with mean 200.  The byte-length table stands in for the
reference's ``token_bytes.pt`` (``prepare.py:200-403``): specials have 0 bytes, every
other id a seeded length uniform in [1, 8].

The generator itself is the native ``_native.BestFitPacker``; this module also holds
a pure-Python mirror (same xoshiro256** stream, same inverse-CDF sampling) that the
tests use to pin the native output bit for bit.
"""
from __future__ import annotations

import math
from bisect import bisect_right

import torch

BOS_ID = 0
N_SPECIAL = 1          # only BOS (id 0) is a special; it counts 0 bytes
ZIPF_S = 1.1
MEAN_DOC_LEN = 200.0
TRAIN_SEED = 1234
VAL_SEED = 987654321
BYTES_SEED = 4242

_M64 = (1 << 64) - 1


def _rotl(x: int, k: int) -> int:
    return ((x << k) | (x >> (64 - k))) & _M64


class PyXoshiro:
    """xoshiro256** seeded via SplitMix64 (pure Python mirror of the native RNG)."""

    def __init__(self, seed: int):
        s = seed & _M64
        self.s = []
        for _ in range(4):
            s = (s + 0x9E3779B97F4A7C15) & _M64
            z = s
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
            self.s.append(z ^ (z >> 31))

    def next(self) -> int:
        s = self.s
        result = (_rotl((s[1] * 5) & _M64, 7) * 9) & _M64
        t = (s[1] << 17) & _M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = _rotl(s[3], 45)
        return result

    def uniform(self) -> float:
        return (self.next() >> 11) * (1.0 / 9007199254740992.0)


class PyZipfDocSource:
    def __init__(self, vocab: int, s: float, mean_doc_len: float, seed: int, bos: int = BOS_ID):
        self.rng = PyXoshiro(seed)
        self.bos = bos
        acc = 0.0
        cdf = []
        for k in range(1, vocab):
            acc += float(k) ** (-s)
            cdf.append(acc)
        self.cdf = [c / acc for c in cdf]
        self.cdf[-1] = 1.0
        p = 1.0 / max(1.0, mean_doc_len)
        self.log1mp = math.log1p(-p)

    def sample_token(self) -> int:
        u = self.rng.uniform()
        idx = bisect_right(self.cdf, u)
        return min(idx, len(self.cdf) - 1) + 1

    def sample_len(self) -> int:
        u = self.rng.uniform()
        if u <= 0.0:
            u = 1e-300
        g = math.floor(math.log(u) / self.log1mp)
        return 1 + int(min(g, 1e7))

    def next_doc(self) -> list[int]:
        n = self.sample_len()
        return [self.bos] + [self.sample_token() for _ in range(n)]


def py_token_bytes(vocab: int, seed: int = BYTES_SEED, lo: int = 1, hi: int = 8,
                   n_special: int = N_SPECIAL) -> torch.Tensor:
    rng = PyXoshiro(seed)
    span = hi - lo + 1
    out = []
    for i in range(vocab):
        r = rng.next()
        out.append(0 if i < n_special else lo + (r % span))
    return torch.tensor(out, dtype=torch.int32)


def rank_seed(base: int, rank: int) -> int:
    """Independent stream per rank (the reference strides row groups by rank;
    with a synthetic source a per-rank seed gives the same disjointness)."""
    return (base * 1000003 + 7919 * (rank + 1)) & _M64


def native():
    from .. import _native_ext
    return _native_ext()


def get_token_bytes(device: torch.device | str = "cpu", vocab: int = 8192) -> torch.Tensor:
    """Per-token byte lengths (int32), specials 0; same role as prepare.get_token_bytes."""
    t = native().token_bytes_table(vocab, BYTES_SEED, 1, 8, N_SPECIAL)
    return t.to(device)


class SyntheticTokenizer:
    """Stand-in for the reference ``Tokenizer`` on the synthetic corpus: exposes the
    BOS id and vocab size that the loaders and the eval harness need."""

    def __init__(self, vocab_size: int = 8192):
        self.vocab_size = vocab_size

    def get_bos_token_id(self) -> int:
        return BOS_ID

    def get_vocab_size(self) -> int:
        return self.vocab_size
