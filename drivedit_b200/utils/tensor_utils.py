"""Tensor helpers (reference ``utils/tensor_utils.py`` :11-321)."""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Union

import torch
import torch.nn.functional as F


def safe_cat(tensors: List[torch.Tensor], dim: int = 0) -> torch.Tensor:
    tensors = [t for t in tensors if t is not None and t.numel() > 0]
    return torch.cat(tensors, dim) if tensors else torch.empty(0)


def safe_stack(tensors: List[torch.Tensor], dim: int = 0) -> torch.Tensor:
    tensors = [t for t in tensors if t is not None]
    return torch.stack(tensors, dim) if tensors else torch.empty(0)


def pad_sequence(sequences: Sequence[torch.Tensor], batch_first: bool = True, padding_value: float = 0.0,
                 max_length: Optional[int] = None) -> torch.Tensor:
    """Pad / truncate along dim 0 and stack (``[B, L, ...]`` or ``[L, B, ...]``); the
    reference's argument order (utils/tensor_utils.py)."""
    if not sequences:
        return torch.empty(0)
    pad_value = padding_value
    L = max_length or max(s.shape[0] for s in sequences)
    out = []
    for s in sequences:
        s = s[:L]
        if s.shape[0] < L:
            s = torch.cat([s, s.new_full((L - s.shape[0],) + tuple(s.shape[1:]), pad_value)], 0)
        out.append(s)
    y = torch.stack(out)
    return y if batch_first else y.transpose(0, 1)


def chunk_tensor(tensor: torch.Tensor, chunk_size: int, dim: int = 1, overlap: int = 0) -> List[torch.Tensor]:
    step = chunk_size - overlap
    assert step > 0
    n = tensor.shape[dim]
    return [tensor.narrow(dim, s, min(chunk_size, n - s)) for s in range(0, max(n - overlap, 1), step)]


def flatten_dict_tensors(tensor_dict: dict, prefix: str = "") -> dict:
    out = {}
    for k, v in tensor_dict.items():
        key = f"{prefix}.{k}" if prefix else k
        if isinstance(v, dict):
            out.update(flatten_dict_tensors(v, key))
        else:
            out[key] = v
    return out


def unflatten_dict_tensors(flattened_dict: dict) -> dict:
    out: Dict[str, Any] = {}
    for k, v in flattened_dict.items():
        d = out
        parts = k.split(".")
        for p in parts[:-1]:
            d = d.setdefault(p, {})
        d[parts[-1]] = v
    return out


def tensor_memory_usage(tensor: torch.Tensor) -> float:
    """MiB."""
    return tensor.numel() * tensor.element_size() / 2 ** 20


def batch_tensor_memory_usage(tensors: List[torch.Tensor]) -> float:
    return sum(tensor_memory_usage(t) for t in tensors if torch.is_tensor(t))


def move_to_device(obj: Any, device, non_blocking: bool = True) -> Any:
    if torch.is_tensor(obj):
        return obj.to(device, non_blocking=non_blocking)
    if isinstance(obj, dict):
        return {k: move_to_device(v, device, non_blocking) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(move_to_device(v, device, non_blocking) for v in obj)
    return obj


def detach_tensors(obj: Any) -> Any:
    if torch.is_tensor(obj):
        return obj.detach()
    if isinstance(obj, dict):
        return {k: detach_tensors(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(detach_tensors(v) for v in obj)
    return obj


def interpolate_tensors(tensor1: torch.Tensor, tensor2: torch.Tensor, alpha: Union[float, torch.Tensor]) -> torch.Tensor:
    return torch.lerp(tensor1, tensor2, alpha if torch.is_tensor(alpha) else float(alpha))


def normalize_tensor(x: torch.Tensor, dim=None, eps: float = 1e-8, mode: str = "l2") -> torch.Tensor:
    """``x / (||x|| + eps)`` over ``dim`` (all elements when None), the reference's
    default; ``mode`` ``minmax`` or ``zscore`` rescale instead."""
    if mode == "l2":
        n = x.norm() if dim is None else x.norm(dim=dim, keepdim=True)
        return x / (n + eps)
    if mode == "minmax":
        lo = x.amin(dim=dim, keepdim=True) if dim is not None else x.min()
        hi = x.amax(dim=dim, keepdim=True) if dim is not None else x.max()
        return (x - lo) / (hi - lo + eps)
    if mode == "zscore":
        m = x.mean(dim=dim, keepdim=True) if dim is not None else x.mean()
        s = x.std(dim=dim, keepdim=True) if dim is not None else x.std()
        return (x - m) / (s + eps)
    raise ValueError(mode)
