"""Unified trainer (flow matching + REPA + C-JEPA + MoE monitor + HASTE + checkpoints), CPU."""
import torch

from drivedit_b200.training.unified import (HASTEController, MoEMonitor, MoEConfig, OnExpertImbalanceCallback,
                                            OnREPADisabledCallback, REPAConfig, TrainingConfig,
                                            UnifiedTrainer, create_training_config)


def _batches(n, B=2, F=4, A=2, rgb=True):
    g = torch.Generator().manual_seed(0)
    out = []
    for _ in range(n):
        b = {"latents": torch.randn(B, F, 16, 16, 16, generator=g), "actions": torch.rand(B, F, A, generator=g)}
        if rgb:
            b["rgb"] = torch.rand(B, F, 3, 64, 64, generator=g)
        out.append(b)
    return out


def test_haste_plateau_and_callbacks():
    fired = []
    h = HASTEController(REPAConfig(enabled=True, haste_warmup_steps=0, haste_window_size=5, haste_patience=2,
                                   haste_threshold=0.01))
    h.add_callback(OnREPADisabledCallback(lambda s, l, t: fired.append(s)))
    active = [h.update(s, 1.0 / (1 + s) if s < 10 else 0.05) for s in range(40)]
    assert not all(active) and fired and h.disable_step == fired[0]
    mon = MoEMonitor(MoEConfig(enabled=True, num_experts=4, top_k=1))
    hits = []
    mon.add_callback(OnExpertImbalanceCallback(0.3, lambda s, u: hits.append(s)))
    logits = torch.tensor([[[10.0, 0, 0, 0]]]).expand(2, 8, 4)
    mon.update(logits, "l0")
    assert mon.check_imbalance(7) and hits == [7]
    assert float(mon.compute_router_z_loss(logits)) > 0


def test_unified_trainer_full_stack(tmp_path):
    from drivedit_b200.config import MoEParams, get_config
    from drivedit_b200.models.world_dit import WorldDiT
    torch.manual_seed(0)
    cfg = get_config("tiny", ["model.n_layers=2", "model.mlp_hidden=0"])
    cfg.model.moe = MoEParams(num_experts=4, top_k=2, expert_dim=64, num_shared=1, aux_loss_weight=0.01)
    tc = create_training_config("full", learning_rate=1e-3, warmup_steps=1, max_steps=100, log_every=2,
                                checkpoint_every=3, checkpoint_dir=str(tmp_path / "ck"), log_dir=str(tmp_path / "log"),
                                initial_sequence_length=2, final_sequence_length=4, curriculum_warmup_steps=4)
    tc.repa.alignment_dim = 64
    tc.repa.projection_hidden_dim = 64
    tc.repa.feature_layer = 1
    tc.cjepa.num_object_queries = 4
    tc.cjepa.object_dim = 32
    tc.cjepa.prediction_horizon = 1
    tc.cjepa.feature_layer = 1
    tc.moe.num_experts = 4
    tr = UnifiedTrainer(WorldDiT(cfg.model), tc, device="cpu")
    res = tr.train_epoch(_batches(6))
    assert {"flow_matching", "repa", "cjepa", "moe_aux", "total"} <= set(res)
    assert tr.global_step == 6 and tr.curriculum.get_sequence_length() == 4
    assert tr.moe_monitor.get_expert_utilization()
    assert (tmp_path / "log" / "metrics.jsonl").exists()
    ev = tr.evaluate(_batches(2))
    assert "val_flow_matching" in ev
    tr2 = UnifiedTrainer(WorldDiT(cfg.model), tc, device="cpu")
    assert tr2.load_checkpoint() and tr2.global_step == 6
    w = dict(tr.model.named_parameters())
    for n, p in tr2.model.named_parameters():
        assert torch.equal(p, w[n]), n
    assert TrainingConfig().is_component_enabled("repa") is False
