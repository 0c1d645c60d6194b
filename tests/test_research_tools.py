"""Research tooling on CPU: checkpoint averaging, summary parsing of the experiment
runner, the evaluation reconciliation plan and a very short autoresearch run."""
import torch


def test_average_checkpoints_selftest_and_refusals(tmp_path):
    from trainium_frontier_b200.research import average_checkpoints as av
    av._selftest()
    a, b = tmp_path / "a.pt", tmp_path / "b.pt"
    cfg = {"n_layer": 1}
    torch.save({"model_state": {"w": torch.ones(2)}, "model_config": cfg, "toggles": {}, "meta": {}}, a)
    torch.save({"model_state": {"w": torch.ones(2)}, "model_config": {"n_layer": 2}, "toggles": {}, "meta": {}}, b)
    try:
        av.average_checkpoints([a, b])
        raise AssertionError("config mismatch accepted")
    except ValueError:
        pass
    try:
        av.average_checkpoints([a, a], "ema")
        raise AssertionError("missing ema accepted")
    except ValueError:
        pass


def test_parse_summary():
    from trainium_frontier_b200.research.run_experiment import parse_summary
    text = "step 00001 | loss 9.0\n---\nval_bpb: 1.234500\ncausality_passed: True\nsteps: 12\nnote with space: x\n"
    s = parse_summary(text)
    assert s == {"val_bpb": 1.2345, "causality_passed": True, "steps": 12}


def test_reconcile_plan():
    from trainium_frontier_b200.research.reconcile_eval import plan_cells
    cells = plan_cells(["short:raw:512"])
    assert [c["name"] for c in cells] == ["raw-2048", "ema-2048", "raw-1024", "ema-1024", "short"]


def test_autoresearch_short_run(tmp_path, capsys):
    from trainium_frontier_b200.research.autoresearch import main
    main(["--time-budget", "1", "--depth", "2", "--n-embd", "128", "--head-dim", "64", "--seq-len", "128",
          "--device-batch-size", "2", "--total-batch-size", "256", "--eval-tokens", "512",
          "--out-dir", str(tmp_path), "--device-type", "cpu"])
    out = capsys.readouterr().out
    assert "val_bpb:" in out and (tmp_path / "final.pt").exists()


def test_op_census_cpu(capsys):
    from trainium_frontier_b200.utils.op_census import main, op_class
    assert op_class("mm") == "matmul" and op_class("view") == "view" and op_class("mul") == "elementwise"
    res = main(["--preset", "tiny", "--depth", "2", "--device", "cpu", "--warmup", "0"])
    assert set(res) == {"fwd_bwd", "sync_clip", "optimizer"}
    # 2 blocks x (q, k, v, proj, fc, proj) forward GEMMs plus the lm_head, and their backward
    assert res["fwd_bwd"]["aten_matmul"] >= 13
    # Newton-Schulz runs on the tensor path
    assert res["optimizer"]["aten_matmul"] > 0
    assert "launch-bound" in capsys.readouterr().out
