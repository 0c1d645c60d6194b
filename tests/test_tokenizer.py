"""Text tokenizer (CPU): BPE training, round trips, BOS prepend, token-byte table,
SHA-verified save / load and archive loading."""
import hashlib
import os
import random
import zipfile

import pytest
import torch

from trainium_frontier_b200.data.tokenizer import SPECIAL_TOKENS, Tokenizer, train_bpe


_LEX = None


def _lexicon():
    """A few thousand made-up words (Zipf-weighted when sampled) plus some fixed ones."""
    global _LEX
    if _LEX is None:
        rnd = random.Random(1234)
        made = ["".join(rnd.choice("etaoinshrdlucmfwypvbgkqjxz") for _ in range(rnd.randint(2, 9)))
                for _ in range(3000)]
        _LEX = ["the", "model", "token", "gradient", "über", "naïve", "日本", "42", "3.14", "don't", "we'll"] + made
    return _LEX


def _corpus(n=400, seed=0):
    rnd = random.Random(seed)
    lex = _lexicon()
    weights = [1.0 / (i + 1) for i in range(len(lex))]
    return [" ".join(rnd.choices(lex, weights, k=rnd.randint(5, 30))) + rnd.choice([".", "!", "\n"])
            for _ in range(n)]


@pytest.fixture(scope="module")
def tok():
    return train_bpe(_corpus(), vocab_size=600)


def test_train_vocab_and_specials(tok):
    assert tok.get_vocab_size() == 600
    assert tok.get_bos_token_id() == 596  # the four reserved tokens sit above the merges
    assert [tok.enc.encode_single_token(t) for t in SPECIAL_TOKENS] == [596, 597, 598, 599]


def test_round_trip_and_prepend(tok):
    for text in _corpus(20, seed=1) + ["", "plain ASCII", "mixed 日本 über 123456"]:
        ids = tok.encode(text)
        assert tok.decode(ids) == text
        assert tok.encode(text, prepend=tok.get_bos_token_id())[0] == tok.get_bos_token_id()
        assert tok.encode(text, prepend=SPECIAL_TOKENS[0])[1:] == ids
    batch = _corpus(8, seed=2)
    rows = tok.encode(batch, prepend=tok.get_bos_token_id(), num_threads=2)
    assert [tok.decode(r[1:]) for r in rows] == batch
    # merges were learned: frequent words compress below one token per byte
    text = " ".join(_corpus(50, seed=3))
    assert len(tok.encode(text)) < 0.5 * len(text.encode("utf-8"))


def test_token_bytes(tok):
    tb = tok.token_bytes()
    assert tb.dtype == torch.int32 and tb.numel() == 600
    assert all(int(tb[tok.enc.encode_single_token(t)]) == 0 for t in SPECIAL_TOKENS)
    text = " ".join(_corpus(30, seed=4))
    assert int(tb[torch.tensor(tok.encode(text))].sum()) == len(text.encode("utf-8"))


def test_training_is_deterministic():
    a = train_bpe(_corpus(200, seed=5), vocab_size=400)
    b = train_bpe(_corpus(200, seed=5), vocab_size=400)
    text = " ".join(_corpus(10, seed=6))
    assert a.encode(text) == b.encode(text)


def test_save_load_verified(tok, tmp_path):
    tok.save(tmp_path)
    sha = hashlib.sha256((tmp_path / "tokenizer.pkl").read_bytes()).hexdigest()
    back = Tokenizer.from_directory(tmp_path, expected_sha=sha, expected_vocab=600)
    text = "the kernel streams memory"
    assert back.encode(text) == tok.encode(text)
    assert torch.equal(back.token_bytes(), tok.token_bytes())
    with pytest.raises(RuntimeError):
        Tokenizer.from_directory(tmp_path, expected_sha="0" * 64, expected_vocab=600)
    with pytest.raises(RuntimeError):
        Tokenizer.from_directory(tmp_path, expected_sha="", expected_vocab=600)
    with pytest.raises(ValueError):
        Tokenizer.from_directory(tmp_path, expected_sha=sha, expected_vocab=8192)


def test_from_zip(tok, tmp_path):
    src = tmp_path / "src"
    tok.save(src)
    archive = tmp_path / "tok.zip"
    with zipfile.ZipFile(archive, "w") as z:
        z.write(src / "tokenizer.pkl", "tokenizer/tokenizer.pkl")
        z.write(src / "token_bytes.pt", "tokenizer/token_bytes.pt")
    sha = lambda p: hashlib.sha256(p.read_bytes()).hexdigest()  # noqa: E731
    with pytest.raises(RuntimeError):
        Tokenizer.from_zip(archive, tmp_path / "cache", expected_sha="1" * 64)
    back = Tokenizer.from_zip(archive, tmp_path / "cache", expected_sha=sha(archive),
                              pkl_sha=sha(src / "tokenizer.pkl"), token_bytes_sha=sha(src / "token_bytes.pt"),
                              expected_vocab=600)
    assert back.decode(back.encode("über naïve")) == "über naïve"


@pytest.mark.skipif(not os.environ.get("TFB_TOKENIZER_ZIP"), reason="set TFB_TOKENIZER_ZIP to the 8192-token artifact")
def test_trusted_artifact(tmp_path):
    tok = Tokenizer.from_zip(os.environ["TFB_TOKENIZER_ZIP"], tmp_path)
    assert tok.get_vocab_size() == 8192
    text = "Hello world, this is a test."
    assert tok.decode(tok.encode(text)) == text


def test_harness_ensure_tokenizer(tok, tmp_path):
    """The harness's setup step verifies and unpacks a named archive (none: nothing to do)."""
    from trainium_frontier_b200.harness import ensure_tokenizer
    assert ensure_tokenizer(tmp_path, None) is None
    src = tmp_path / "src"
    tok.save(src)
    archive = tmp_path / "tok.zip"
    with zipfile.ZipFile(archive, "w") as z:
        z.write(src / "tokenizer.pkl", "tokenizer.pkl")
        z.write(src / "token_bytes.pt", "token_bytes.pt")
    sha = lambda p: hashlib.sha256(p.read_bytes()).hexdigest()  # noqa: E731
    back = ensure_tokenizer(tmp_path / "cache", archive, expected_sha=sha(archive), pkl_sha=sha(src / "tokenizer.pkl"),
                            token_bytes_sha=sha(src / "token_bytes.pt"), expected_vocab=600)
    assert (tmp_path / "cache" / "tokenizer" / "tokenizer.pkl").exists()
    assert back.encode("the model") == tok.encode("the model")
    with pytest.raises(RuntimeError):
        ensure_tokenizer(tmp_path / "cache2", archive)  # the trusted pins do not match this archive
