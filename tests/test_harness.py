"""Harness CLI (setup / check / eval-public) and the static submission rules, on CPU."""
import json
import os
import sys

import pytest

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_check_accepts_own_train_script():
    from trainium_frontier_b200.harness import check_submission
    path = os.path.join(ROOT, "trainium_frontier_b200", "train.py")
    assert check_submission(path) == []
    ok = "torchrun --standalone --nproc-per-node 8 train.py"
    assert check_submission(path, ok) == []


def test_check_flags_forbidden_code(tmp_path):
    from trainium_frontier_b200.harness import check_submission
    p = tmp_path / "train.py"
    p.write_text("import socket\nfrom subprocess import run\nimport os\nos.system('x')\neval('1')\n")
    w = check_submission(str(p))
    assert any("forbidden import: socket" in x for x in w)
    assert any("forbidden import: subprocess" in x for x in w)
    assert any("os.system" in x for x in w)
    assert any("eval()" in x for x in w)
    assert any("record_step_boundary" in x for x in w)


def test_launch_command_rules(tmp_path):
    from trainium_frontier_b200.harness import launch_command_warnings
    assert launch_command_warnings("torchrun --nproc_per_node=4 train.py", "train.py") == []
    assert launch_command_warnings("python train.py --depth 4", "train.py") == []
    assert launch_command_warnings("torchrun --nproc-per-node 3 train.py", "train.py")
    assert launch_command_warnings("torchrun --nproc-per-node 8 train.py; rm -rf x", "train.py")
    assert launch_command_warnings("bash train.py", "train.py")
    assert launch_command_warnings("torchrun --nproc-per-node 8 other.py", "train.py")


def test_setup_manifest_is_stable(tmp_path):
    from trainium_frontier_b200.harness import ensure_data
    a = ensure_data(tmp_path, stream_tokens=4096)
    b = ensure_data(tmp_path, stream_tokens=4096)   # verifies against the stored manifest
    assert a == b and (tmp_path / "token_bytes.pt").exists()
    assert set(a["splits"]) == {"train", "public_val"}


def test_eval_public_cli(tmp_path, capsys):
    from trainium_frontier_b200.checkpoint import save_checkpoint
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.harness import main
    from trainium_frontier_b200.models.gpt import GPT
    cfg = preset("tiny", depth=2)
    torch.manual_seed(0)
    m = GPT(cfg.model_config(), cfg)
    m.init_weights()
    ck = tmp_path / "final.pt"
    save_checkpoint(ck, m, {"step": 0})
    script = tmp_path / "train.py"
    script.write_text(f"import sys\nsys.path.insert(0, {ROOT!r})\n"
                      "from trainium_frontier_b200.checkpoint import load_for_eval\n")
    main(["eval-public", "--train-py", str(script), "--checkpoint", str(ck), "--device", "cpu",
          "--batch-size", "2", "--seq-len", "128", "--eval-tokens", "1024"])
    out = json.loads(capsys.readouterr().out)
    assert out["num_tokens"] >= 1024 and 0 < out["val_bpb"] < 10


def test_eval_public_on_held_out_text(tmp_path, capsys):
    """eval-public --text-val-data: the checkpoint is scored on held-out parquet text
    tokenized with the verified archive, bytes from the tokenizer's UTF-8 table."""
    import hashlib
    import random
    import zipfile
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from trainium_frontier_b200.checkpoint import save_checkpoint
    from trainium_frontier_b200.config import preset
    from trainium_frontier_b200.data.tokenizer import train_bpe
    from trainium_frontier_b200.harness import main
    from trainium_frontier_b200.models.gpt import GPT
    rnd = random.Random(0)
    words = ["alpha", "beta", "gamma", "tensor", "core", "kernel", "memory", "über", "42"]
    docs = [" ".join(rnd.choice(words) for _ in range(rnd.randint(5, 40))) for _ in range(200)]
    tok = train_bpe(docs, vocab_size=300)
    src = tmp_path / "tok"
    tok.save(src)
    archive = tmp_path / "tok.zip"
    with zipfile.ZipFile(archive, "w") as z:
        z.write(src / "tokenizer.pkl", "tokenizer.pkl")
        z.write(src / "token_bytes.pt", "token_bytes.pt")
    sha = lambda p: hashlib.sha256(p.read_bytes()).hexdigest()  # noqa: E731
    os.environ["NEURON_COMPETITION_R1_TOKENIZER_SHA256"] = sha(archive)
    os.environ["NEURON_COMPETITION_R1_TOKENIZER_PKL_SHA256"] = sha(src / "tokenizer.pkl")
    os.environ["NEURON_COMPETITION_R1_TOKEN_BYTES_SHA256"] = sha(src / "token_bytes.pt")
    try:
        pq.write_table(pa.table({"text": docs}), tmp_path / "val.parquet", row_group_size=50)
        cfg = preset("tiny", depth=2, vocab_size=tok.get_vocab_size())
        torch.manual_seed(0)
        m = GPT(cfg.model_config(), cfg)
        m.init_weights()
        ck = tmp_path / "final.pt"
        save_checkpoint(ck, m, {"step": 0})
        script = tmp_path / "train.py"
        script.write_text(f"import sys\nsys.path.insert(0, {ROOT!r})\n"
                          "from trainium_frontier_b200.checkpoint import load_for_eval\n")
        main(["eval-public", "--train-py", str(script), "--checkpoint", str(ck), "--device", "cpu",
              "--batch-size", "2", "--seq-len", "128", "--eval-tokens", "512",
              "--text-val-data", str(tmp_path / "val.parquet"), "--tokenizer-zip", str(archive),
              "--cache-dir", str(tmp_path / "cache")])
    finally:
        for k in ("NEURON_COMPETITION_R1_TOKENIZER_SHA256", "NEURON_COMPETITION_R1_TOKENIZER_PKL_SHA256",
                  "NEURON_COMPETITION_R1_TOKEN_BYTES_SHA256"):
            os.environ.pop(k, None)
    out = json.loads(capsys.readouterr().out)
    assert out["num_tokens"] >= 512 and out["num_bytes"] > out["num_tokens"] and out["val_bpb"] > 0
