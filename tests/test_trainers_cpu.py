"""Self-forcing (first generation) and teacher -> student distillation trainers on CPU."""
import torch

from drivedit_b200.config.presets import ModelConfig
from drivedit_b200.models.world_dit import WorldDiT
from drivedit_b200.training.distill import DistillationTrainer
from drivedit_b200.training.self_forcing_v1 import (SelfForcingTrainer, create_dummy_dataloader,
                                                    create_simple_model)


def test_self_forcing_v1_trains_and_checkpoints(tmp_path):
    torch.manual_seed(0)
    model = create_simple_model(hidden_dim=32)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    tr = SelfForcingTrainer(model, opt, checkpoint_dir=str(tmp_path), mixed_precision=False,
                            checkpoint_every=2, context_length=2, prediction_horizon=3)
    dl = create_dummy_dataloader(batch_size=2, num_batches=2, frames=6, size=16)
    first = tr.train_epoch(dl)
    for _ in range(4):
        last = tr.train_epoch(dl)
    assert last["total"] < first["total"]
    assert set(first) >= {"reconstruction", "temporal_consistency", "perceptual", "total"}
    v = tr.validate(dl)
    assert v["total"] > 0
    info = tr.load_checkpoint()
    assert info["step"] == 10 and tr.get_training_stats()["global_step"] == 10


def test_distillation_student_learns_teacher_endpoint():
    torch.manual_seed(0)
    ms = ModelConfig(n_layers=2, d_model=64, n_heads=2, mlp_hidden=128, latent_channels=4,
                     latent_h=8, latent_w=8)
    mt = ModelConfig(n_layers=4, d_model=96, n_heads=2, mlp_hidden=128, latent_channels=4,
                     latent_h=8, latent_w=8, causal="none")
    student, teacher = WorldDiT(ms), WorldDiT(mt)
    with torch.no_grad():                   # a teacher with a non-trivial velocity field
        teacher.out_proj.weight.normal_(0, 0.05)
    opt = torch.optim.AdamW(student.parameters(), lr=2e-3)
    tr = DistillationTrainer(teacher, student, None, opt, device="cpu")
    g = torch.Generator().manual_seed(1)
    batch = {"latents": torch.randn(2, 3, 4, 8, 8, generator=g), "controls": torch.rand(2, 3, 2, generator=g)}
    before = tr.validate([batch])["one_step_endpoint_mse"]
    hist = [tr.train_step(batch) for _ in range(30)]
    after = tr.validate([batch])["one_step_endpoint_mse"]
    assert set(hist[0]) == {"flow_matching", "kl_divergence", "consistency", "feature_matching", "total"}
    assert after < before
    assert hist[-1]["flow_matching"] < hist[0]["flow_matching"]
