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


def test_piecewise_schedule_shapes_period_and_restart():
    from drivedit_b200.utils.schedules import PiecewiseSchedule, Segment, ramp

    assert ramp(0.5, "linear") == 0.5 and abs(ramp(0.5, "cosine") - 0.5) < 1e-12
    assert ramp(0.99, "step") == 0.0 and ramp(1.0, "step") == 1.0
    s = PiecewiseSchedule([Segment(10, 0.0, 1.0, "linear", "up"),
                           Segment(None, 1.0, 1.0, "constant", "hold")])
    assert s(0) == 0.0 and s(5) == 0.5 and s(10) == 1.0 and s(10 ** 6) == 1.0
    assert s.phase(3) == "up" and s.phase(11) == "hold"
    cyc = PiecewiseSchedule([Segment(4, 0.0, 1.0, "linear")], period=4)
    assert [cyc(i) for i in range(6)] == [0.0, 0.25, 0.5, 0.75, 0.0, 0.25]
    cyc.restart(5)
    assert cyc(5) == 0.0 and cyc(7) == 0.5


def test_haste_step_shape_switches_on_at_the_end_of_warmup():
    from drivedit_b200.training.repa import HASTEScheduler, REPAConfig

    h = HASTEScheduler(REPAConfig(total_training_steps=100, haste_warmup_ratio=0.1,
                                  haste_termination_ratio=0.5, haste_schedule="step"))
    assert [h.get_weight(s) for s in (0, 5, 9, 10, 49, 50)] == [0.0, 0.0, 0.0, 1.0, 1.0, 0.0]
    assert h.get_phase() == "terminated"


def test_uncertainty_weighting_matches_the_kendall_objective():
    import torch

    from drivedit_b200.training.self_forcing import UncertaintyWeighting

    uw = UncertaintyWeighting(["a", "b", "c"], initial_log_var=0.3)
    with torch.no_grad():
        uw.log_vars.copy_(torch.tensor([0.1, -0.4, 2.0]))
    la, lb = torch.tensor(2.0), torch.tensor(0.5)
    total, w = uw({"a": la, "b": lb})
    s = uw.log_vars.detach()
    expect = 0.5 * (torch.exp(-s[0]) * la + s[0]) + 0.5 * (torch.exp(-s[1]) * lb + s[1])
    assert torch.allclose(total, expect) and set(w) == {"a", "b"}
    total.backward()
    assert uw.log_vars.grad[2] == 0.0  # an absent task gets no gradient
