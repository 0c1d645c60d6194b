"""Text training rows (CPU): tokenized documents packed BOS-aligned best-fit by the
native DocPacker, from an iterable of strings or from parquet row groups."""
import random

import pytest
import torch

from trainium_frontier_b200.data.text_loader import parquet_documents, text_dataloader
from trainium_frontier_b200.data.tokenizer import train_bpe


def _docs(n, seed=0):
    rnd = random.Random(seed)
    words = ["alpha", "beta", "gamma", "delta", "tensor", "core", "über", "42", "kernel", "memory"]
    return [f"doc{i} " + " ".join(rnd.choice(words) for _ in range(rnd.randint(3, 60))) for i in range(n)]


@pytest.fixture(scope="module")
def tok():
    return train_bpe(_docs(300, seed=7), vocab_size=400)


def test_rows_are_bos_aligned_documents(tok):
    docs = _docs(2000)
    T = 128
    batches = list(text_dataloader(tok, docs, batch_size=4, seq_len=T, buffer_min=32))
    assert batches, "no rows"
    bos = tok.get_bos_token_id()
    encoded = {tuple(tok.encode(d)) for d in docs}
    whole = 0
    for x, y in batches:
        assert x.dtype == torch.int32 and y.dtype == torch.int64 and x.shape == (4, T) and y.shape == (4, T)
        assert torch.equal(x[:, 1:].long(), y[:, :-1])
        for row in torch.cat([x, y[:, -1:].int()], 1).tolist():
            assert row[0] == bos  # every row starts with a document
            # split at BOS: every piece is a document, whole or (the last one) cropped
            starts = [i for i, t in enumerate(row) if t == bos]
            for a, b in zip(starts, starts[1:] + [len(row)]):
                piece = tuple(row[a + 1:b])
                if b < len(row):
                    assert piece in encoded
                    whole += 1
                else:
                    assert any(e[:len(piece)] == piece for e in encoded)
    assert whole > 0


def test_rank_striding_and_end_of_data(tok):
    docs = _docs(400, seed=3)
    T = 64
    seen = []
    for r in range(2):
        n = 0
        for x, _ in text_dataloader(tok, docs, batch_size=2, seq_len=T, rank=r, world=2, buffer_min=8):
            n += x.shape[0]
            seen.append(x)
        assert n > 0
    # the two ranks' first rows differ (different documents)
    assert not torch.equal(seen[0], seen[-1])


def test_parquet_documents(tok, tmp_path):
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    docs = _docs(300, seed=5)
    path = tmp_path / "shard.parquet"
    pq.write_table(pa.table({"text": docs}), path, row_group_size=50)
    assert list(parquet_documents([path])) == docs
    r0 = list(parquet_documents([path], rank=0, world=2))
    r1 = list(parquet_documents([path], rank=1, world=2))
    assert sorted(r0 + r1) == sorted(docs) and len(r0) == 150  # 6 row groups, alternating
    x, y = next(text_dataloader(tok, parquet_documents([path]), batch_size=2, seq_len=64, buffer_min=16))
    assert x[0, 0] == tok.get_bos_token_id()


def test_trainer_on_text_files(tok, tmp_path, monkeypatch):
    """--text-data / --tokenizer-zip: the trainer packs rows from parquet text tokenized
    with the verified archive (epochs repeat when the files run out) and takes steps."""
    import hashlib
    import zipfile
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.train import Trainer
    for i in range(2):
        pq.write_table(pa.table({"text": _docs(150, seed=20 + i)}), tmp_path / f"s{i}.parquet", row_group_size=30)
    src = tmp_path / "tok"
    tok.save(src)
    archive = tmp_path / "tok.zip"
    with zipfile.ZipFile(archive, "w") as z:
        z.write(src / "tokenizer.pkl", "tokenizer.pkl")
        z.write(src / "token_bytes.pt", "token_bytes.pt")
    sha = lambda p: hashlib.sha256(p.read_bytes()).hexdigest()  # noqa: E731
    monkeypatch.setenv("NEURON_COMPETITION_R1_TOKENIZER_SHA256", sha(archive))
    monkeypatch.setenv("NEURON_COMPETITION_R1_TOKENIZER_PKL_SHA256", sha(src / "tokenizer.pkl"))
    monkeypatch.setenv("NEURON_COMPETITION_R1_TOKEN_BYTES_SHA256", sha(src / "token_bytes.pt"))
    monkeypatch.setenv("NEURON_COMPETITION_R1_CACHE_DIR", str(tmp_path / "cache"))
    V = tok.get_vocab_size()
    pq.write_table(pa.table({"text": _docs(60, seed=99)}), tmp_path / "val.parquet", row_group_size=20)
    cfg = preset("tiny", depth=2, n_embd=128, head_dim=64, seq_len=64, vocab_size=V, device_batch_size=2,
                 total_batch_size=2 * 64, progress_mode="steps", num_steps=5, text_data=str(tmp_path / "s*.parquet"),
                 tokenizer_zip=str(archive), text_val_data=str(tmp_path / "val.parquet"))
    tr = Trainer(cfg, torch.device("cpu"))
    rows = tr.loader.next()
    assert rows.shape == (2, 65) and int(rows[0, 0]) == tok.get_bos_token_id() and int(rows.max()) < V
    losses = [tr.train_step() for _ in range(3)]
    assert all(l == l for l in losses)
    for _ in range(40):  # well past one epoch of the two small files
        tr.loader.next()
    assert tr.loader.packer.epoch >= 1
    # the final evaluation scores the held-out text with its UTF-8 byte lengths
    from trainium_frontier_b200.data.loader import make_eval_dataloader
    from trainium_frontier_b200.eval import evaluate_bpb
    etok = tr.eval_tokenizer()
    x, y, _ = next(make_eval_dataloader(etok, 2, 64, "public_val", "cpu", max_stream_tokens=4096))
    assert int(x[0, 0]) == tok.get_bos_token_id()
    res = evaluate_bpb(tr.model, etok, 2, 64, "cpu", max_tokens=1024)
    assert 0 < res["val_bpb"] < 100 and res["num_bytes"] > res["num_tokens"]  # multi-byte tokens
