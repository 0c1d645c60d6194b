"""Text tokenizer: a wrapper over a tiktoken BPE encoding with the reference's interface,
SHA-verified loading of the trusted artifact, a token-byte table, and a byte-level BPE
trainer for building an encoding without the artifact.

* ``Tokenizer(enc)`` - ``encode(text | [texts], prepend=None, num_threads=8)`` (ordinary
  encoding, optional BOS / id prepended to every row), ``decode(ids)``,
  ``get_vocab_size()``, ``get_bos_token_id()``, ``token_bytes()`` (UTF-8 byte length of
  every id, 0 for the special tokens: the bpb denominator).
* ``Tokenizer.from_directory(dir, expected_sha=...)`` loads ``tokenizer.pkl`` (a pickled
  ``tiktoken.Encoding``) only if its SHA-256 matches; ``Tokenizer.from_zip(path, ...)``
  verifies the archive, unpacks ``tokenizer.pkl`` / ``token_bytes.pt`` into a cache
  directory and loads from there.  Verification cannot be skipped (an empty pin raises).
* ``train_bpe(texts, vocab_size)`` - byte-level BPE over the pre-tokenisation split
  pattern: 256 single-byte tokens, then greedy merges of the most frequent adjacent pair
  (ties broken by the smaller pair, so training is deterministic), then the reserved
  special tokens at the top of the vocabulary.  ``save(directory)`` writes
  ``tokenizer.pkl`` and ``token_bytes.pt``.

The pinned hashes, the split pattern, the vocabulary size and the special-token names are
the trusted artifact's identity and stay as the reference defines them (``prepare.py:56-75``);
the wrapper follows ``prepare.py:200-260`` and the artifact loader / fallback builder
``prepare.py:262-403``.  The training pipeline of this framework runs on the seeded
synthetic corpus (``data/synthetic.py``); this module serves text data when it exists.
"""
from __future__ import annotations

import collections
import hashlib
import os
import pickle
import zipfile
from pathlib import Path

import torch

VOCAB_SIZE = 8192
SPECIAL_TOKENS = [f"<|reserved_{i}|>" for i in range(4)]
BOS_TOKEN = SPECIAL_TOKENS[0]
SPLIT_PATTERN = (r"""'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,2}| ?[^\s\p{L}\p{N}]++[\r\n]*|"""
                 r"""\s*[\r\n]|\s+(?!\S)|\s+""")
ARTIFACT_SHA256 = os.environ.get("NEURON_COMPETITION_R1_TOKENIZER_SHA256",
                                 "12fa2c4a56d9f26d46e8ea0a57f69d78145930eecb0a765c9bfc085176af8a54")
PKL_SHA256 = os.environ.get("NEURON_COMPETITION_R1_TOKENIZER_PKL_SHA256",
                            "aacd6c6a838eaec2c662a7d0cba0b5412f930a6ddee95b9ecb2c8fac53f3dafc")
TOKEN_BYTES_SHA256 = os.environ.get("NEURON_COMPETITION_R1_TOKEN_BYTES_SHA256",
                                    "3de03cf6f8e16a9397fecd0cebd04f435f11994b215a5c785787fcc15adb0e15")


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _pin(env: str, default: str, given: str | None) -> str:
    """An explicit hash, else the environment override, else the pinned default."""
    return given if given is not None else os.environ.get(env, default)


def _require_sha(path: Path, expected: str, what: str) -> None:
    if not expected:
        raise RuntimeError(f"refusing to load {path}: no expected SHA-256 for the {what}")
    got = _sha256(path)
    if got != expected:
        raise RuntimeError(f"{what} SHA-256 mismatch at {path}: expected {expected}, got {got}")


class Tokenizer:
    def __init__(self, enc):
        self.enc = enc
        self.bos_token_id = enc.encode_single_token(BOS_TOKEN)
        self._token_bytes = None
        # optional held-out text for evaluate_bpb: a callable (rank, world) -> iterable of str
        self.eval_documents = None

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_directory(cls, directory, *, expected_sha: str | None = None,
                       expected_vocab: int | None = VOCAB_SIZE) -> "Tokenizer":
        """``expected_sha`` None: the pinned hash (or its environment override, read now)."""
        path = Path(directory) / "tokenizer.pkl"
        _require_sha(path, _pin("NEURON_COMPETITION_R1_TOKENIZER_PKL_SHA256", PKL_SHA256, expected_sha),
                     "tokenizer.pkl")
        with open(path, "rb") as f:
            enc = pickle.load(f)
        tok = cls(enc)
        if expected_vocab is not None and tok.get_vocab_size() != expected_vocab:
            raise ValueError(f"expected vocab size {expected_vocab}, got {tok.get_vocab_size()}")
        tb = Path(directory) / "token_bytes.pt"
        if tb.exists():
            tok._token_bytes = torch.load(tb, map_location="cpu", weights_only=True)
        return tok

    @classmethod
    def from_zip(cls, archive, cache_dir, *, expected_sha: str | None = None, pkl_sha: str | None = None,
                 token_bytes_sha: str | None = None, expected_vocab: int | None = VOCAB_SIZE) -> "Tokenizer":
        """Hashes left None: the pinned ones (or their environment overrides, read now)."""
        archive, cache_dir = Path(archive), Path(cache_dir)
        _require_sha(archive, _pin("NEURON_COMPETITION_R1_TOKENIZER_SHA256", ARTIFACT_SHA256, expected_sha),
                     "tokenizer archive")
        cache_dir.mkdir(parents=True, exist_ok=True)
        with zipfile.ZipFile(archive) as z:
            for name in ("tokenizer.pkl", "token_bytes.pt"):
                member = next((m for m in z.namelist() if m.rsplit("/", 1)[-1] == name), None)
                if member is None:
                    raise RuntimeError(f"{archive} has no {name}")
                (cache_dir / name).write_bytes(z.read(member))
        _require_sha(cache_dir / "token_bytes.pt",
                     _pin("NEURON_COMPETITION_R1_TOKEN_BYTES_SHA256", TOKEN_BYTES_SHA256, token_bytes_sha),
                     "token_bytes.pt")
        return cls.from_directory(cache_dir, expected_sha=pkl_sha, expected_vocab=expected_vocab)

    # ------------------------------------------------------------------ interface
    def get_vocab_size(self) -> int:
        return self.enc.n_vocab

    def get_bos_token_id(self) -> int:
        return self.bos_token_id

    def encode(self, text, prepend=None, num_threads: int = 8):
        pid = None
        if prepend is not None:
            pid = prepend if isinstance(prepend, int) else self.enc.encode_single_token(prepend)
        if isinstance(text, str):
            ids = self.enc.encode_ordinary(text)
            return ids if pid is None else [pid] + ids
        if isinstance(text, list):
            rows = self.enc.encode_ordinary_batch(text, num_threads=num_threads)
            return rows if pid is None else [[pid] + r for r in rows]
        raise TypeError(f"unsupported text type: {type(text).__name__}")

    def decode(self, ids) -> str:
        return self.enc.decode(list(ids))

    def token_bytes(self) -> torch.Tensor:
        """int32 [vocab]: UTF-8 byte length of each token, 0 for the special tokens."""
        if self._token_bytes is None:
            special = {self.enc.encode_single_token(t) for t in SPECIAL_TOKENS}
            lens = [0 if i in special else len(self.enc.decode_single_token_bytes(i))
                    for i in range(self.enc.n_vocab)]
            self._token_bytes = torch.tensor(lens, dtype=torch.int32)
        return self._token_bytes

    def save(self, directory) -> None:
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        with open(d / "tokenizer.pkl", "wb") as f:
            pickle.dump(self.enc, f)
        torch.save(self.token_bytes(), d / "token_bytes.pt")


# ---------------------------------------------------------------------- BPE training
def train_bpe(texts, vocab_size: int = VOCAB_SIZE, name: str = "tfb_bpe") -> Tokenizer:
    """Byte-level BPE over the split pattern: up to ``vocab_size - len(SPECIAL_TOKENS) - 256``
    merges of the most frequent adjacent pair (pair counts weighted by pre-token
    frequency, updated incrementally per merge; ties go to the smaller pair).  A corpus
    with fewer distinct pairs yields a smaller vocabulary."""
    import regex
    import tiktoken
    n_merges = vocab_size - len(SPECIAL_TOKENS) - 256
    if n_merges < 0:
        raise ValueError("vocab_size must leave room for the 256 bytes and the special tokens")
    pat = regex.compile(SPLIT_PATTERN)
    words: collections.Counter = collections.Counter()
    for t in texts:
        for piece in pat.findall(t):
            words[piece.encode("utf-8")] += 1
    # each distinct pre-token as a list of token ids, with its frequency
    seqs = [list(w) for w in words]
    freq = list(words.values())
    ranks = {bytes([i]): i for i in range(256)}
    token_of = [bytes([i]) for i in range(256)]
    pairs: collections.Counter = collections.Counter()
    where: dict = collections.defaultdict(set)  # pair -> indices of sequences holding it
    for si, s in enumerate(seqs):
        for a, b in zip(s, s[1:]):
            pairs[(a, b)] += freq[si]
            where[(a, b)].add(si)
    for _ in range(n_merges):
        if not pairs:
            break
        best = max(pairs.items(), key=lambda kv: (kv[1], -kv[0][0], -kv[0][1]))[0]
        if pairs[best] <= 0:
            break
        new_id = len(token_of)
        token_of.append(token_of[best[0]] + token_of[best[1]])
        ranks[token_of[-1]] = new_id
        for si in list(where.pop(best, ())):
            s, f = seqs[si], freq[si]
            for a, b in zip(s, s[1:]):          # remove this sequence's old pair counts
                pairs[(a, b)] -= f
            out, i = [], 0
            while i < len(s):
                if i + 1 < len(s) and s[i] == best[0] and s[i + 1] == best[1]:
                    out.append(new_id)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[si] = out
            for a, b in zip(out, out[1:]):      # and add the new ones
                pairs[(a, b)] += f
                where[(a, b)].add(si)
        pairs.pop(best, None)
        for p in [p for p, c in pairs.items() if c <= 0]:
            del pairs[p]
    n = len(ranks)
    enc = tiktoken.Encoding(name=name, pat_str=SPLIT_PATTERN, mergeable_ranks=ranks,
                            special_tokens={t: n + i for i, t in enumerate(SPECIAL_TOKENS)})
    return Tokenizer(enc)
