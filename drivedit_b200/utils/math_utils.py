"""Math helpers (reference ``utils/math_utils.py`` :12-407)."""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def gaussian_kernel(size: int, sigma: float, device=None) -> torch.Tensor:
    x = torch.arange(size, device=device, dtype=torch.float32) - (size - 1) / 2
    g = torch.exp(-x ** 2 / (2 * sigma ** 2))
    k = g[:, None] * g[None]
    return k / k.sum()


def soft_clamp(x: torch.Tensor, min_val: float = -1.0, max_val: float = 1.0) -> torch.Tensor:
    """Smooth clamp: ``mid + half * tanh((x - mid) / half)``."""
    mid, half = (max_val + min_val) / 2, (max_val - min_val) / 2
    return mid + half * torch.tanh((x - mid) / half)


def stable_softmax(x: torch.Tensor, dim: int = -1, temperature: float = 1.0) -> torch.Tensor:
    z = x / temperature
    return torch.softmax(z - z.amax(dim, keepdim=True), dim)


def log_sum_exp(x: torch.Tensor, dim: int = -1, keepdim: bool = False) -> torch.Tensor:
    return torch.logsumexp(x, dim, keepdim=keepdim)


def gumbel_noise(shape: Tuple[int, ...], device=None, eps: float = 1e-10) -> torch.Tensor:
    u = torch.rand(shape, device=device)
    return -torch.log(-torch.log(u + eps) + eps)


def gumbel_softmax(logits: torch.Tensor, temperature: float = 1.0, hard: bool = False, dim: int = -1) -> torch.Tensor:
    y = torch.softmax((logits + gumbel_noise(logits.shape, logits.device)) / temperature, dim)
    if not hard:
        return y
    idx = y.argmax(dim, keepdim=True)
    y_hard = torch.zeros_like(y).scatter_(dim, idx, 1.0)
    return y_hard - y.detach() + y


def cosine_similarity_matrix(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return F.normalize(x, dim=-1) @ F.normalize(y, dim=-1).transpose(-1, -2)


def pairwise_distance_matrix(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return torch.cdist(x, y)


def smoothing_kernel(size: int, smoothing_type: str = "gaussian") -> torch.Tensor:
    if smoothing_type == "gaussian":
        x = torch.arange(size, dtype=torch.float32) - (size - 1) / 2
        k = torch.exp(-x ** 2 / (2 * (size / 4) ** 2))
    elif smoothing_type == "uniform":
        k = torch.ones(size)
    elif smoothing_type == "triangular":
        k = 1 - (torch.arange(size, dtype=torch.float32) - (size - 1) / 2).abs() / ((size + 1) / 2)
    else:
        raise ValueError(smoothing_type)
    return k / k.sum()


def finite_difference_gradient(x: torch.Tensor, spacing: float = 1.0,
                               edge_order: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
    """Spatial gradients ``(d/dy, d/dx)`` over the last two dims of ``x [..., H, W]``
    (utils/math_utils.py:194-231): central differences inside and one-sided ones at the
    borders with ``edge_order=1``; periodic central differences (wrapping at the
    borders) otherwise."""
    if edge_order == 1:
        gy, gx = torch.gradient(x, spacing=spacing, dim=(-2, -1), edge_order=1)
        return gy, gx
    return ((x.roll(-1, -2) - x.roll(1, -2)) / (2 * spacing),
            (x.roll(-1, -1) - x.roll(1, -1)) / (2 * spacing))


def gradient_along(x: torch.Tensor, dim: int = -1, spacing: float = 1.0, order: int = 1) -> torch.Tensor:
    """``order``-th derivative along one dim: central differences inside, one-sided at
    the ends (``torch.gradient`` applied ``order`` times)."""
    g = x
    for _ in range(order):
        g = torch.gradient(g, spacing=spacing, dim=dim)[0]
    return g


def laplacian(x: torch.Tensor, spacing: float = 1.0) -> torch.Tensor:
    """5-point Laplacian over the last two dims."""
    k = torch.tensor([[0, 1, 0], [1, -4, 1], [0, 1, 0]], dtype=x.dtype, device=x.device) / spacing ** 2
    s = x.shape
    y = F.conv2d(x.reshape(-1, 1, s[-2], s[-1]), k[None, None], padding=1)
    return y.view(s)


def spectral_norm_power_iteration(weight: torch.Tensor, u: Optional[torch.Tensor] = None,
                                  num_iterations: int = 1) -> Tuple[torch.Tensor, torch.Tensor]:
    """Power iteration for the largest singular value of ``weight [out, in]`` from the
    left-vector estimate ``u`` (random when None): returns ``(u, sigma)`` with ``u``
    updated, to be passed back in on the next call (utils/math_utils.py)."""
    with torch.no_grad():
        if u is None:
            u = F.normalize(torch.randn(weight.shape[0], device=weight.device, dtype=weight.dtype), dim=0)
        v = F.normalize(weight.t() @ u, dim=0, eps=1e-12)
        for _ in range(num_iterations):
            v = F.normalize(weight.t() @ u, dim=0, eps=1e-12)
            u = F.normalize(weight @ v, dim=0, eps=1e-12)
        return u, u @ weight @ v


def batch_trace(x: torch.Tensor) -> torch.Tensor:
    return x.diagonal(dim1=-2, dim2=-1).sum(-1)


def batch_determinant(x: torch.Tensor) -> torch.Tensor:
    return torch.linalg.det(x)


def matrix_sqrt(x: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """Symmetric PSD square root by eigendecomposition."""
    e, v = torch.linalg.eigh(x)
    return v @ torch.diag_embed(e.clamp_min(eps).sqrt()) @ v.transpose(-1, -2)


def frechet_distance(mu1, sigma1, mu2, sigma2) -> torch.Tensor:
    r1 = matrix_sqrt(sigma1.double(), 0.0)
    m = r1 @ sigma2.double() @ r1
    tr = torch.linalg.eigvalsh((m + m.T) / 2).clamp_min(0).sqrt().sum()
    return ((mu1 - mu2).double().pow(2).sum() + torch.trace(sigma1.double()) + torch.trace(sigma2.double())
            - 2 * tr).float()


def wasserstein_distance_1d(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """W1 between two equal-size 1-D empirical distributions (sorted differences)."""
    return (x.flatten().sort().values - y.flatten().sort().values).abs().mean()


def sinkhorn_divergence(x: torch.Tensor, y: torch.Tensor, reg: float = 0.1, num_iters: int = 100) -> torch.Tensor:
    """Entropic OT cost (log-domain Sinkhorn) debiased: ``OT(x,y) - (OT(x,x)+OT(y,y))/2``."""
    def ot(a, b):
        C = torch.cdist(a, b) ** 2
        n, m = C.shape
        la, lb = torch.full((n,), -math.log(n), device=a.device), torch.full((m,), -math.log(m), device=a.device)
        f, g = torch.zeros(n, device=a.device), torch.zeros(m, device=a.device)
        for _ in range(num_iters):
            f = -reg * torch.logsumexp((g[None] - C) / reg + lb[None], 1)
            g = -reg * torch.logsumexp((f[:, None] - C) / reg + la[:, None], 0)
        P = torch.exp((f[:, None] + g[None] - C) / reg + la[:, None] + lb[None])
        return (P * C).sum()
    return ot(x, y) - 0.5 * (ot(x, x) + ot(y, y))
