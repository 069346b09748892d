"""Generic training helpers on CPU (the GPU-only pieces degrade to plain calls)."""
import torch
import torch.nn as nn
from torch.utils.data import TensorDataset

from drivedit_b200.training.cuda_optimized import (AsyncPrefetcher, CUDAControlNormalizer, CUDADataPipeline,
                                                   CUDAOptimizedConfig, GradientAccumulator, OptimizedTrainer,
                                                   create_cosine_scheduler, create_optimized_optimizer)


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = nn.Linear(8, 8)
        self.norm = nn.LayerNorm(8)

    def forward(self, x, y=None):
        return self.norm(self.lin(x))


def test_trainer_accumulates_and_learns(tmp_path):
    torch.manual_seed(0)
    net = _Net()
    cfg = CUDAOptimizedConfig(gradient_accumulation_steps=2, num_workers=0)
    tr = OptimizedTrainer(net, cfg, torch.device("cpu"))
    opt = create_optimized_optimizer(net, lr=1e-2)
    assert len(opt.param_groups) == 2 and opt.param_groups[1]["weight_decay"] == 0.0
    sched = create_cosine_scheduler(opt, total_steps=20, warmup_steps=2)
    x = torch.randn(16, 8)
    y = torch.randn(16, 8)
    loss_fn = lambda out, b: {"total": ((out - b["y"]) ** 2).mean()}
    data = [{"x": x, "y": y}] * 10
    first = tr.train_step(data[0], opt, loss_fn)
    assert first["stepped"] == 0.0
    ep = tr.train_epoch(data, opt, loss_fn, sched)
    assert ep["loss"] < first["loss"]
    tr.save_checkpoint(str(tmp_path / "c.pt"), opt, sched)
    assert tr.load_checkpoint(str(tmp_path / "c.pt"), opt, sched)["global_step"] == 11
    assert tr.validate_step(data[0], loss_fn)["val_loss"] > 0


def test_pipeline_normalizer_accumulator():
    ds = TensorDataset(torch.arange(12.0).view(6, 2))
    pipe = CUDADataPipeline(ds, 2, CUDAOptimizedConfig(num_workers=0), device=torch.device("cpu"), shuffle=False)
    assert [b[0][0, 0].item() for b in pipe] == [0.0, 4.0, 8.0]
    assert len(list(AsyncPrefetcher([1, 2, 3], torch.device("cpu"), 2))) == 3
    n = CUDAControlNormalizer(3, momentum=1.0)
    c = torch.randn(10, 4, 3) * 5 + 2
    out = n(c)
    assert abs(float(out.mean())) < 1e-4 and abs(float(out.std()) - 1.0) < 0.05
    n.set_ego_transform(torch.tensor([[1., 0, 0, 1], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1]]))
    assert torch.allclose(n.transform_ego(torch.zeros(2, 3)), torch.tensor([[1., 0, 0]] * 2))
    acc = GradientAccumulator(3)
    assert [acc.step() for _ in range(6)] == [False, False, True, False, False, True]
    assert float(acc.scale_loss(torch.tensor(3.0))) == 1.0
