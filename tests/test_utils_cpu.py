"""Profiling helpers that need no GPU."""
import os


def test_dead_code_report_lists_unreferenced_definitions(tmp_path):
    from drivedit_b200.profiling import StepProfile, dead_code

    (tmp_path / "a.py").write_text("def used():\n    return 1\n\ndef orphan_fn():\n    return used()\n")
    (tmp_path / "b.py").write_text("from a import used\nclass Lonely:\n    pass\n")
    out = dead_code(str(tmp_path))
    assert any("orphan_fn" in o for o in out) and any("Lonely" in o for o in out)
    assert not any(o.endswith(" used") for o in out)
    p = StepProfile("x", 2.0, 1000.0, [{"name": "k", "calls": 3, "total_ms": 1.5, "share": 0.75}])
    assert "75.0%" in p.table()


def test_cli_train_resume(tmp_path):
    import json

    from drivedit_b200.cli import main

    out = tmp_path / "run"
    assert main(["train", "--config", "tiny", "--steps", "2", "--log-every", "1", "--ckpt-every", "2",
                 "--out", str(out), "model.n_layers=1"]) == 0
    assert main(["train", "--config", "tiny", "--steps", "3", "--log-every", "1", "--out", str(out), "--resume",
                 "model.n_layers=1"]) == 0
    steps = [json.loads(l)["step"] for l in (out / "metrics.jsonl").read_text().splitlines()]
    assert steps == [1, 2, 3]
