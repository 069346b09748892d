"""Video / latent / temporal / control / depth / physics / perceptual metrics.

Same metric families and names as the reference ``evaluation/metrics.py``
(``VideoMetrics`` :13-114, ``LatentMetrics`` :117-163, ``TemporalConsistencyMetrics``
:166-262, ``ControlMetrics`` :265-310, ``DepthMetrics`` :313-355, ``PhysicsMetrics``
:358-432, ``PerceptualMetrics`` :435-478, ``compute_all_metrics`` :481). Video tensors
are ``[B, T, C, H, W]`` (or ``[N, C, H, W]``) in [0, 1]. All metrics are batched tensor
ops (GPU friendly); none synchronises with the host.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn.functional as F


def _frames(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, *x.shape[-3:]) if x.dim() == 5 else x


class VideoMetrics:
    @staticmethod
    def mse(pred, target, mask: Optional[torch.Tensor] = None):
        d = (pred.float() - target.float()) ** 2
        return (d * mask).sum() / mask.sum().clamp_min(1) if mask is not None else d.mean()

    @staticmethod
    def mae(pred, target, mask: Optional[torch.Tensor] = None):
        d = (pred.float() - target.float()).abs()
        return (d * mask).sum() / mask.sum().clamp_min(1) if mask is not None else d.mean()

    @staticmethod
    def psnr(pred, target, max_val: float = 1.0):
        p, t = _frames(pred).float(), _frames(target).float()
        mse = ((p - t) ** 2).flatten(1).mean(1)
        return (10 * torch.log10(max_val ** 2 / mse.clamp_min(1e-12))).mean()

    @staticmethod
    def ssim(pred, target, window_size: int = 11, max_val: float = 1.0):
        """Gaussian-window SSIM (Wang et al. 2004), averaged over frames and channels."""
        p, t = _frames(pred).float(), _frames(target).float()
        C = p.shape[1]
        sigma = 1.5
        g = torch.exp(-(torch.arange(window_size, device=p.device) - window_size // 2).float() ** 2 / (2 * sigma ** 2))
        g = g / g.sum()
        w = (g[:, None] * g[None, :])[None, None].expand(C, 1, window_size, window_size)
        pad = window_size // 2
        mu_p = F.conv2d(p, w, padding=pad, groups=C)
        mu_t = F.conv2d(t, w, padding=pad, groups=C)
        s_pp = F.conv2d(p * p, w, padding=pad, groups=C) - mu_p ** 2
        s_tt = F.conv2d(t * t, w, padding=pad, groups=C) - mu_t ** 2
        s_pt = F.conv2d(p * t, w, padding=pad, groups=C) - mu_p * mu_t
        c1, c2 = (0.01 * max_val) ** 2, (0.03 * max_val) ** 2
        m = ((2 * mu_p * mu_t + c1) * (2 * s_pt + c2)) / ((mu_p ** 2 + mu_t ** 2 + c1) * (s_pp + s_tt + c2))
        return m.mean()

    @staticmethod
    def lpips_proxy(pred, target):
        """Distance between multi-scale gradient / intensity features (a learned-
        feature-free stand-in for LPIPS; no pretrained network is available offline)."""
        def feats(x):
            out = []
            for _ in range(3):
                gx = x[..., :, 1:] - x[..., :, :-1]
                gy = x[..., 1:, :] - x[..., :-1, :]
                out += [x.flatten(1), gx.flatten(1), gy.flatten(1)]
                x = F.avg_pool2d(x, 2)
            return out
        fp, ft = feats(_frames(pred).float()), feats(_frames(target).float())
        return torch.stack([F.mse_loss(a, b) for a, b in zip(fp, ft)]).mean()


class LatentMetrics:
    @staticmethod
    def latent_mse(pred_latents, target_latents):
        return F.mse_loss(pred_latents.float(), target_latents.float())

    @staticmethod
    def latent_cosine_similarity(pred_latents, target_latents):
        return F.cosine_similarity(pred_latents.float().flatten(1), target_latents.float().flatten(1), dim=1).mean()

    @staticmethod
    def latent_diversity(latents):
        """Mean pairwise distance between samples of the batch."""
        z = latents.float().flatten(1)
        d = torch.cdist(z, z)
        n = z.shape[0]
        return d.sum() / max(n * (n - 1), 1)

    @staticmethod
    def latent_smoothness(latents):
        """Mean squared difference between consecutive frames ``[B, T, ...]``."""
        return (latents[:, 1:].float() - latents[:, :-1].float()).pow(2).mean()

    @staticmethod
    def latent_reconstruction_error(latents, reconstructed):
        return F.mse_loss(reconstructed.float(), latents.float())


class TemporalConsistencyMetrics:
    @staticmethod
    def temporal_mse(frames):
        return (frames[:, 1:].float() - frames[:, :-1].float()).pow(2).mean()

    @staticmethod
    def _compute_simple_flow(frames):
        """Per-pixel flow from image gradients and the temporal difference (one
        Lucas-Kanade step without windowing): ``[B, T-1, 2, H, W]``."""
        g = frames.float().mean(2)                                  # [B, T, H, W]
        It = g[:, 1:] - g[:, :-1]
        Ix = F.pad(g[:, :-1, :, 1:] - g[:, :-1, :, :-1], (0, 1))
        Iy = F.pad(g[:, :-1, 1:, :] - g[:, :-1, :-1, :], (0, 0, 0, 1))
        den = Ix ** 2 + Iy ** 2 + 1e-3
        return torch.stack([-It * Ix / den, -It * Iy / den], 2)

    @staticmethod
    def _warp_frames(frames, flows):
        """Warp frame t by flow t -> prediction of frame t+1."""
        B, T1, _, H, W = flows.shape
        src = frames[:, :-1].float().reshape(B * T1, -1, H, W)
        fl = flows.reshape(B * T1, 2, H, W)
        yy, xx = torch.meshgrid(torch.arange(H, device=frames.device), torch.arange(W, device=frames.device),
                                indexing="ij")
        gx = (xx[None] - fl[:, 0]) / max(W - 1, 1) * 2 - 1
        gy = (yy[None] - fl[:, 1]) / max(H - 1, 1) * 2 - 1
        out = F.grid_sample(src, torch.stack([gx, gy], -1), align_corners=True, padding_mode="border")
        return out.reshape(B, T1, -1, H, W)

    @classmethod
    def optical_flow_consistency(cls, frames):
        """Smoothness of the estimated flow field over time (lower = steadier motion)."""
        fl = cls._compute_simple_flow(frames)
        return (fl[:, 1:] - fl[:, :-1]).pow(2).mean() if fl.shape[1] > 1 else fl.new_zeros(())

    @classmethod
    def frame_warping_error(cls, frames, flows: Optional[torch.Tensor] = None):
        fl = cls._compute_simple_flow(frames) if flows is None else flows
        return (cls._warp_frames(frames, fl) - frames[:, 1:].float()).abs().mean()


class ControlMetrics:
    @staticmethod
    def control_mse(pred_controls, target_controls):
        return F.mse_loss(pred_controls.float(), target_controls.float())

    @staticmethod
    def control_mae(pred_controls, target_controls):
        return F.l1_loss(pred_controls.float(), target_controls.float())

    @staticmethod
    def steering_accuracy(pred_controls, target_controls, threshold: float = 0.1):
        return ((pred_controls[..., 0] - target_controls[..., 0]).abs() < threshold).float().mean()

    @staticmethod
    def acceleration_accuracy(pred_controls, target_controls, threshold: float = 0.1):
        return ((pred_controls[..., 1] - target_controls[..., 1]).abs() < threshold).float().mean()

    @staticmethod
    def control_smoothness(controls):
        """Mean squared second difference over time (lower = smoother)."""
        d2 = controls[:, 2:].float() - 2 * controls[:, 1:-1].float() + controls[:, :-2].float()
        return d2.pow(2).mean()


class DepthMetrics:
    @staticmethod
    def _m(x, mask):
        return (x * mask).sum() / mask.sum().clamp_min(1) if mask is not None else x.mean()

    @classmethod
    def depth_mse(cls, pred_depth, target_depth, mask=None):
        return cls._m((pred_depth.float() - target_depth.float()) ** 2, mask)

    @classmethod
    def depth_mae(cls, pred_depth, target_depth, mask=None):
        return cls._m((pred_depth.float() - target_depth.float()).abs(), mask)

    @classmethod
    def depth_relative_error(cls, pred_depth, target_depth, mask=None):
        t = target_depth.float()
        return cls._m((pred_depth.float() - t).abs() / t.abs().clamp_min(1e-6), mask)

    @staticmethod
    def depth_gradient_consistency(depth):
        d = depth.float()
        return ((d[..., 1:, :] - d[..., :-1, :]).abs().mean() + (d[..., :, 1:] - d[..., :, :-1]).abs().mean()) / 2


class PhysicsMetrics:
    """Trajectories ``[B, T, 2]`` (x, y)."""

    @staticmethod
    def trajectory_smoothness(positions):
        acc = positions[:, 2:] - 2 * positions[:, 1:-1] + positions[:, :-2]
        return acc.float().norm(dim=-1).mean()

    @staticmethod
    def speed_consistency(positions, dt: float = 1.0):
        speed = (positions[:, 1:] - positions[:, :-1]).float().norm(dim=-1) / dt
        return speed.std(dim=1).mean() if speed.shape[1] > 1 else speed.new_zeros(())

    @staticmethod
    def _compute_turning_validity(positions, min_radius: float):
        a, b, c = positions[:, :-2].float(), positions[:, 1:-1].float(), positions[:, 2:].float()
        ab, bc, ca = (b - a).norm(dim=-1), (c - b).norm(dim=-1), (a - c).norm(dim=-1)
        cross = ((b - a)[..., 0] * (c - a)[..., 1] - (b - a)[..., 1] * (c - a)[..., 0]).abs()
        radius = ab * bc * ca / (2 * cross).clamp_min(1e-9)     # circumradius of the 3 points
        return (radius >= min_radius).float().mean()

    @classmethod
    def turning_radius_validity(cls, positions, min_radius: float = 1.0):
        if positions.shape[1] < 3:
            return positions.new_ones(())
        return cls._compute_turning_validity(positions, min_radius)


class PerceptualMetrics:
    @staticmethod
    def feature_matching_distance(pred_features, target_features):
        return (pred_features.float().mean(0) - target_features.float().mean(0)).norm()

    @staticmethod
    def frechet_distance(pred_features, target_features):
        """Fréchet distance between Gaussians fitted to two feature sets ``[N, D]``
        (the FID / FVD formula; the trace term through the eigenvalues of
        ``S1^1/2 S2 S1^1/2``)."""
        a, b = pred_features.double(), target_features.double()
        mu1, mu2 = a.mean(0), b.mean(0)
        s1, s2 = torch.cov(a.T), torch.cov(b.T)
        e, v = torch.linalg.eigh(s1)
        r1 = v @ torch.diag(e.clamp_min(0).sqrt()) @ v.T
        m = r1 @ s2 @ r1
        tr = torch.linalg.eigvalsh((m + m.T) / 2).clamp_min(0).sqrt().sum()
        return ((mu1 - mu2).pow(2).sum() + torch.trace(s1) + torch.trace(s2) - 2 * tr).float()

    @staticmethod
    def inception_score(features, epsilon: float = 1e-16):
        """``exp(E_x KL(p(y|x) || p(y)))`` from class probabilities ``[N, K]``."""
        p = features.float().softmax(-1) if (features < 0).any() or (features.sum(-1) - 1).abs().max() > 1e-3 \
            else features.float()
        py = p.mean(0, keepdim=True)
        kl = (p * ((p + epsilon).log() - (py + epsilon).log())).sum(-1)
        return kl.mean().exp()


def compute_all_metrics(pred_frames: torch.Tensor, target_frames: torch.Tensor, pred_controls=None,
                        target_controls=None, pred_depth=None, target_depth=None,
                        positions=None) -> Dict[str, torch.Tensor]:
    """Frame, temporal, control, depth and trajectory metrics (the reference's argument
    names, evaluation/metrics.py)."""
    pred, target = pred_frames, target_frames
    m: Dict[str, torch.Tensor] = {
        "mse": VideoMetrics.mse(pred, target), "mae": VideoMetrics.mae(pred, target),
        "psnr": VideoMetrics.psnr(pred, target), "ssim": VideoMetrics.ssim(pred, target),
        "lpips_proxy": VideoMetrics.lpips_proxy(pred, target),
    }
    if pred.dim() == 5 and pred.shape[1] > 1:
        m["temporal_mse"] = TemporalConsistencyMetrics.temporal_mse(pred)
        m["warping_error"] = TemporalConsistencyMetrics.frame_warping_error(pred)
    if pred_controls is not None and target_controls is not None:
        m["control_mse"] = ControlMetrics.control_mse(pred_controls, target_controls)
        m["steering_accuracy"] = ControlMetrics.steering_accuracy(pred_controls, target_controls)
    if pred_depth is not None and target_depth is not None:
        m["depth_mae"] = DepthMetrics.depth_mae(pred_depth, target_depth)
    if positions is not None:
        m["trajectory_smoothness"] = PhysicsMetrics.trajectory_smoothness(positions)
    return m
