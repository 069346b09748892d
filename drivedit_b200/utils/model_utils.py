"""Model helpers (reference ``utils/model_utils.py`` :13-414): parameter counting,
freezing, seeding, init, gradient norms (device-side), checkpoint save / load with the
reference's dict keys, EMA, summaries, layer lookup / replacement."""
from __future__ import annotations

import random
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn


def count_parameters(model: nn.Module, trainable_only: bool = True) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad or not trainable_only)


def freeze_parameters(model: nn.Module, freeze: bool = True) -> None:
    for p in model.parameters():
        p.requires_grad = not freeze


def freeze_layers(model: nn.Module, layer_names: List[str]) -> None:
    for n, p in model.named_parameters():
        if any(n.startswith(l) for l in layer_names):
            p.requires_grad = False


def get_device(model: nn.Module) -> torch.device:
    for p in model.parameters():
        return p.device
    for b in model.buffers():
        return b.device
    return torch.device("cpu")


def get_model_size_mb(model: nn.Module) -> float:
    return (sum(p.numel() * p.element_size() for p in model.parameters())
            + sum(b.numel() * b.element_size() for b in model.buffers())) / 2 ** 20


def set_seed(seed: int) -> None:
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def initialize_weights(model: nn.Module, init_type: str = "normal", gain: float = 0.02) -> None:
    for m in model.modules():
        if isinstance(m, (nn.Linear, nn.Conv1d, nn.Conv2d, nn.Conv3d)):
            if init_type == "normal":
                nn.init.normal_(m.weight, 0.0, gain)
            elif init_type == "xavier":
                nn.init.xavier_normal_(m.weight, gain=gain)
            elif init_type == "kaiming":
                nn.init.kaiming_normal_(m.weight, a=0, mode="fan_in")
            elif init_type == "orthogonal":
                nn.init.orthogonal_(m.weight, gain=gain)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, (nn.LayerNorm, nn.GroupNorm, nn.BatchNorm1d, nn.BatchNorm2d)) and m.weight is not None:
            nn.init.ones_(m.weight)
            nn.init.zeros_(m.bias)


def get_gradient_norm(model: nn.Module) -> torch.Tensor:
    """Global L2 norm of all gradients as a device tensor (no host sync)."""
    g = [p.grad for p in model.parameters() if p.grad is not None]
    if not g:
        return torch.zeros(())
    return torch.stack(torch._foreach_norm(g)).float().norm()


def clip_gradients(model: nn.Module, max_norm: float = 1.0) -> torch.Tensor:
    return torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm, foreach=True)


def save_checkpoint(model: nn.Module, optimizer, epoch: int, loss: float, filepath: str, scheduler=None,
                    **kwargs) -> None:
    ck = {"epoch": epoch, "model_state_dict": model.state_dict(),
          "optimizer_state_dict": optimizer.state_dict() if optimizer is not None else None,
          "loss": float(loss), **kwargs}
    if scheduler is not None:
        ck["scheduler_state_dict"] = scheduler.state_dict()
    torch.save(ck, filepath)


def load_checkpoint(filepath: str, model: nn.Module, optimizer=None, scheduler=None, device=None,
                    strict: bool = True) -> Dict[str, Any]:
    ck = torch.load(filepath, map_location=device)
    sd = ck.get("model_state_dict", ck.get("model", ck))
    model.load_state_dict(sd, strict=strict)
    if optimizer is not None and ck.get("optimizer_state_dict") is not None:
        optimizer.load_state_dict(ck["optimizer_state_dict"])
    if scheduler is not None and ck.get("scheduler_state_dict") is not None:
        scheduler.load_state_dict(ck["scheduler_state_dict"])
    return ck


@torch.no_grad()
def exponential_moving_average(model: nn.Module, ema_model: nn.Module, decay: float = 0.999) -> None:
    """``ema <- decay * ema + (1 - decay) * model`` for every parameter (the reference's
    argument order, utils/model_utils.py:241-258: the live model first)."""
    ep, mp = list(ema_model.parameters()), list(model.parameters())
    torch._foreach_lerp_(ep, [p.detach() for p in mp], 1 - decay)


def model_summary(model: nn.Module, input_size: Optional[Tuple[int, ...]] = None) -> str:
    lines = [f"{'module':60s} {'params':>14s}"]
    for n, m in model.named_modules():
        own = sum(p.numel() for p in m.parameters(recurse=False))
        if own:
            lines.append(f"{n or '(root)':60s} {own:14,d}")
    lines.append(f"{'total':60s} {count_parameters(model, False):14,d}")
    lines.append(f"{'trainable':60s} {count_parameters(model, True):14,d}")
    lines.append(f"{'size (MiB)':60s} {get_model_size_mb(model):14.2f}")
    return "\n".join(lines)


def compare_models(model1: nn.Module, model2: nn.Module) -> Dict[str, bool]:
    a, b = model1.state_dict(), model2.state_dict()
    return {k: (k in b and a[k].shape == b[k].shape and torch.equal(a[k].cpu(), b[k].cpu())) for k in a}


def get_layer_by_name(model: nn.Module, layer_name: str) -> nn.Module:
    m = model
    for p in layer_name.split("."):
        m = m[int(p)] if p.isdigit() else getattr(m, p)
    return m


def replace_layer(model: nn.Module, layer_name: str, new_layer: nn.Module) -> None:
    parts = layer_name.split(".")
    parent = get_layer_by_name(model, ".".join(parts[:-1])) if len(parts) > 1 else model
    if parts[-1].isdigit():
        parent[int(parts[-1])] = new_layer
    else:
        setattr(parent, parts[-1], new_layer)
