"""GAIA-2-style rich conditioning: camera, road topology, 3-D boxes, ego state, time and
weather -> one global conditioning vector, AdaLN modulation parameters and
cross-attention contexts, with classifier-free-guidance dropout.

Same capabilities and call contract as the reference's ``models/conditioning.py``
(enums :29-65, ``ConditioningConfig`` :68-102, encoders :193-1083, ``AdaLNModulation``
:1090-1132, ``ConditioningIntegration`` :1135-1440, factory :1447-1481): the
``forward`` takes per-modality dicts and returns ``{'conditioning', 'adaln_params',
'road_context', 'object_tokens', 'modality_mask'}``. Missing modalities are replaced by
learned null tokens, which is also what CFG dropout substitutes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class ObjectClass(Enum):
    VEHICLE = 0
    PEDESTRIAN = 1
    CYCLIST = 2
    MOTORCYCLE = 3
    TRUCK = 4
    BUS = 5
    TRAILER = 6
    CONSTRUCTION = 7
    TRAFFIC_SIGN = 8
    TRAFFIC_LIGHT = 9
    OTHER = 10


class RoadType(Enum):
    HIGHWAY = 0
    URBAN = 1
    RURAL = 2
    INTERSECTION = 3
    ROUNDABOUT = 4
    PARKING = 5
    OFFRAMP = 6
    ONRAMP = 7


class WeatherCondition(Enum):
    CLEAR = 0
    CLOUDY = 1
    RAIN = 2
    SNOW = 3
    FOG = 4
    NIGHT = 5
    DUSK = 6
    DAWN = 7


@dataclass
class ConditioningConfig:
    model_dim: int = 512
    cond_dim: int = 256
    num_cameras: int = 6
    camera_embed_dim: int = 128
    max_waypoints: int = 50
    max_lanes: int = 8
    road_embed_dim: int = 128
    road_cross_attn_heads: int = 4
    max_objects: int = 64
    bbox_embed_dim: int = 128
    num_object_classes: int = 11
    ego_state_dim: int = 64
    time_embed_dim: int = 64
    weather_embed_dim: int = 32
    num_adaln_modulation_outputs: int = 6
    dropout: float = 0.1
    cfg_dropout_prob: float = 0.1
    image_size: Tuple[int, int] = (256, 512)  # addition: normalises the camera intrinsics


def normalize_intrinsics(K: torch.Tensor, image_size: Tuple[int, int]) -> torch.Tensor:
    """Focal lengths / principal point divided by the image width/height."""
    H, W = image_size
    Kn = K.clone().float()
    Kn[..., 0, :] = Kn[..., 0, :] / W
    Kn[..., 1, :] = Kn[..., 1, :] / H
    return Kn


def rotation_matrix_to_6d(R: torch.Tensor) -> torch.Tensor:
    """Continuous 6-D rotation representation: the first two columns (Zhou et al. 2019)."""
    return torch.cat([R[..., :, 0], R[..., :, 1]], -1)


def sinusoidal_embedding(x: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=x.device, dtype=torch.float32) / half)
    ang = x.float()[..., None] * freqs
    emb = torch.cat([ang.sin(), ang.cos()], -1)
    return F.pad(emb, (0, dim % 2))


def _mlp(i, h, o, drop=0.0):
    return nn.Sequential(nn.Linear(i, h), nn.SiLU(), nn.Dropout(drop), nn.Linear(h, o))


class CameraEncoder(nn.Module):
    """Intrinsics (fx, fy, cx, cy, skew) + extrinsics (6-D rotation, translation) + a
    camera-id embedding -> per-camera tokens, mean-pooled to one vector."""

    def __init__(self, embed_dim: int = 128, output_dim: int = 256, num_cameras: int = 6,
                 image_size: Tuple[int, int] = (256, 512), dropout: float = 0.0):
        super().__init__()
        self.image_size = image_size
        self.camera_embed = nn.Embedding(num_cameras, embed_dim)
        self.proj = _mlp(5 + 9 + embed_dim, embed_dim * 2, output_dim, dropout)

    def forward(self, intrinsics, extrinsics, camera_ids=None, return_per_camera: bool = False):
        B, N = intrinsics.shape[:2]
        K = normalize_intrinsics(intrinsics, self.image_size)
        intr = torch.stack([K[..., 0, 0], K[..., 1, 1], K[..., 0, 2], K[..., 1, 2], K[..., 0, 1]], -1)
        extr = torch.cat([rotation_matrix_to_6d(extrinsics[..., :3, :3].float()), extrinsics[..., :3, 3].float()], -1)
        ids = camera_ids if camera_ids is not None else torch.arange(N, device=intrinsics.device)[None].expand(B, N)
        tok = self.proj(torch.cat([intr, extr, self.camera_embed(ids)], -1))
        return tok if return_per_camera else tok.mean(1)


class RoadTopologyEncoder(nn.Module):
    """Waypoints (x, y, z, heading, curvature, speed limit) -> tokens; road type, lane and
    turn features -> a global vector; returns (global [B, D], context tokens [B, N, D])."""

    def __init__(self, embed_dim: int = 128, output_dim: int = 256, max_waypoints: int = 50,
                 max_lanes: int = 8, num_road_types: int = 8, num_heads: int = 4, dropout: float = 0.0):
        super().__init__()
        self.max_waypoints, self.max_lanes = max_waypoints, max_lanes
        self.wp_proj = _mlp(6 + 32, embed_dim, output_dim, dropout)
        self.road_type = nn.Embedding(num_road_types, output_dim)
        self.lane_proj = nn.Linear(3, output_dim)
        self.turn_proj = nn.Linear(5, output_dim)
        self.encoder = nn.TransformerEncoder(
            nn.TransformerEncoderLayer(output_dim, num_heads, 2 * output_dim, batch_first=True,
                                       norm_first=True), 1, enable_nested_tensor=False)
        self.cross_attn = nn.MultiheadAttention(output_dim, num_heads, batch_first=True)
        self.out = nn.Linear(output_dim, output_dim)

    def forward(self, waypoints, road_type, lane_info, turn_info=None, waypoint_mask=None):
        B, N = waypoints.shape[:2]
        idx = sinusoidal_embedding(torch.arange(N, device=waypoints.device), 32)[None].expand(B, N, 32)
        tok = self.wp_proj(torch.cat([waypoints.float(), idx], -1))
        pad = None if waypoint_mask is None else ~waypoint_mask.bool()
        tok = self.encoder(tok, src_key_padding_mask=pad)
        if waypoint_mask is not None:
            w = waypoint_mask.float()[..., None]
            pooled = (tok * w).sum(1) / w.sum(1).clamp(min=1)
        else:
            pooled = tok.mean(1)
        g = pooled + self.road_type(road_type.long()) + self.lane_proj(lane_info.float())
        if turn_info is not None:
            g = g + self.turn_proj(turn_info.float())
        return self.out(g), tok

    def apply_cross_attention(self, x: torch.Tensor, context: torch.Tensor, mask=None):
        pad = None if mask is None else ~mask.bool()
        return self.cross_attn(x, context, context, key_padding_mask=pad)[0]


class BoundingBox3DEncoder(nn.Module):
    """Per-object (position, size, heading sin/cos, velocity, confidence, class) tokens,
    distance-weighted pooling (closer objects count more); returns (global, tokens)."""

    def __init__(self, embed_dim: int = 128, output_dim: int = 256, max_objects: int = 64,
                 num_object_classes: int = 11, num_heads: int = 4, dropout: float = 0.0):
        super().__init__()
        self.max_objects = max_objects
        self.class_embed = nn.Embedding(num_object_classes, embed_dim)
        self.proj = _mlp(3 + 3 + 2 + 3 + 1 + embed_dim, embed_dim * 2, output_dim, dropout)
        self.attn = nn.MultiheadAttention(output_dim, num_heads, batch_first=True)
        self.norm = nn.LayerNorm(output_dim)
        self.out = nn.Linear(output_dim, output_dim)

    def _compute_distance_weights(self, positions, mask=None, scale: float = 20.0):
        w = torch.exp(-positions.float().norm(dim=-1) / scale)
        if mask is not None:
            w = w * mask.float()
        return w / w.sum(-1, keepdim=True).clamp(min=1e-6)

    def forward(self, positions, dimensions, headings, velocities, object_classes, confidences,
                object_mask=None):
        feats = torch.cat([positions.float(), dimensions.float(), headings.sin()[..., None].float(),
                           headings.cos()[..., None].float(), velocities.float(),
                           confidences.float()[..., None], self.class_embed(object_classes.long())], -1)
        tok = self.proj(feats)
        pad = None if object_mask is None else ~object_mask.bool()
        if pad is not None:
            pad = pad.clone()
            pad[pad.all(-1), 0] = False  # keep attention defined when no object is present
        tok = self.norm(tok + self.attn(tok, tok, tok, key_padding_mask=pad)[0])
        w = self._compute_distance_weights(positions, object_mask)
        return self.out((tok * w[..., None]).sum(1)), tok


class EgoStateEncoder(nn.Module):
    """Position, velocity, acceleration, heading (sin/cos), heading rate, optional GPS/IMU."""

    def __init__(self, embed_dim: int = 64, output_dim: int = 256, use_gps: bool = True,
                 use_imu: bool = True, dropout: float = 0.0, gps_dim: int = 3, imu_dim: int = 6):
        super().__init__()
        self.base = _mlp(3 + 3 + 3 + 2 + 1, embed_dim, output_dim, dropout)
        self.gps = nn.Linear(gps_dim, output_dim) if use_gps else None
        self.imu = nn.Linear(imu_dim, output_dim) if use_imu else None

    def forward(self, position, velocity, acceleration, heading, heading_rate, gps=None, imu=None):
        x = torch.cat([position.float(), velocity.float(), acceleration.float(),
                       heading.sin()[..., None].float(), heading.cos()[..., None].float(),
                       heading_rate.float()[..., None]], -1)
        out = self.base(x)
        if gps is not None and self.gps is not None:
            out = out + self.gps(gps.float())
        if imu is not None and self.imu is not None:
            out = out + self.imu(imu.float())
        return out


class TemporalEnvironmentalEncoder(nn.Module):
    """Time of day (cyclic), weather (+ intensity), season, sun angles, lighting."""

    def __init__(self, time_embed_dim: int = 64, weather_embed_dim: int = 32, output_dim: int = 256,
                 num_weather_conditions: int = 8, num_seasons: int = 4, dropout: float = 0.0):
        super().__init__()
        self.weather = nn.Embedding(num_weather_conditions, weather_embed_dim)
        self.season = nn.Embedding(num_seasons, weather_embed_dim)
        self.proj = _mlp(time_embed_dim + 2 * weather_embed_dim + 1 + 4 + 1, output_dim, output_dim, dropout)
        self.time_dim = time_embed_dim

    def forward(self, time_of_day, weather, weather_intensity=None, season=None, sun_azimuth=None,
                sun_elevation=None, lighting=None):
        B = time_of_day.shape[0]
        z = time_of_day.new_zeros(B)
        ang = time_of_day.float() / 24.0 * 2 * math.pi
        t = sinusoidal_embedding(ang, self.time_dim)
        wi = (weather_intensity if weather_intensity is not None else z).float()[:, None]
        se = self.season(season.long()) if season is not None else self.season.weight.new_zeros(B, self.season.embedding_dim)
        az = (sun_azimuth if sun_azimuth is not None else z).float()
        el = (sun_elevation if sun_elevation is not None else z).float()
        li = (lighting if lighting is not None else z).float()[:, None]
        sun = torch.stack([az.sin(), az.cos(), el.sin(), el.cos()], -1)
        return self.proj(torch.cat([t, self.weather(weather.long()), se, wi, sun, li], -1))


class AdaLNModulation(nn.Module):
    """cond -> ``n`` modulation vectors (scale/shift/gate for attention and MLP); zero
    init, so scales and shifts start at 0 and gates at 0 (adaLN-Zero)."""

    def __init__(self, cond_dim: int, model_dim: int, num_outputs: int = 6):
        super().__init__()
        self.num_outputs = num_outputs
        self.proj = nn.Sequential(nn.SiLU(), nn.Linear(cond_dim, num_outputs * model_dim))
        nn.init.zeros_(self.proj[1].weight)
        nn.init.zeros_(self.proj[1].bias)

    def forward(self, conditioning: torch.Tensor) -> Tuple[torch.Tensor, ...]:
        return tuple(self.proj(conditioning).chunk(self.num_outputs, -1))


class ConditioningIntegration(nn.Module):
    MODALITIES = ("camera", "road", "bbox", "ego", "temporal")

    def __init__(self, config: Optional[ConditioningConfig] = None):
        super().__init__()
        c = self.config = config or ConditioningConfig()
        D = c.cond_dim
        self.camera_encoder = CameraEncoder(c.camera_embed_dim, D, c.num_cameras, c.image_size, c.dropout)
        self.road_encoder = RoadTopologyEncoder(c.road_embed_dim, D, c.max_waypoints, c.max_lanes,
                                                num_heads=c.road_cross_attn_heads, dropout=c.dropout)
        self.bbox_encoder = BoundingBox3DEncoder(c.bbox_embed_dim, D, c.max_objects, c.num_object_classes,
                                                 dropout=c.dropout)
        self.ego_encoder = EgoStateEncoder(c.ego_state_dim, D, dropout=c.dropout)
        self.temporal_encoder = TemporalEnvironmentalEncoder(c.time_embed_dim, c.weather_embed_dim, D,
                                                             dropout=c.dropout)
        self.null_tokens = nn.Parameter(torch.zeros(len(self.MODALITIES), D))
        self.fusion = nn.Sequential(nn.Linear(len(self.MODALITIES) * D, 2 * D), nn.SiLU(),
                                    nn.Dropout(c.dropout), nn.Linear(2 * D, D))
        self.norm = nn.LayerNorm(D)
        self.adaln = AdaLNModulation(D, c.model_dim, c.num_adaln_modulation_outputs)
        self.context_proj = nn.Linear(D, c.model_dim)

    def _apply_cfg_dropout(self, emb: torch.Tensor, idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        B = emb.shape[0]
        if self.training and self.config.cfg_dropout_prob > 0:
            keep = (torch.rand(B, device=emb.device) >= self.config.cfg_dropout_prob)
        else:
            keep = torch.ones(B, dtype=torch.bool, device=emb.device)
        return torch.where(keep[:, None], emb, self.null_tokens[idx].expand_as(emb)), keep

    @staticmethod
    def _batch_device(*ds):
        for d in ds:
            if d:
                v = next(iter(d.values()))
                return v.shape[0], v.device
        raise ValueError("at least one conditioning modality is required")

    def forward(self, camera_data=None, road_data=None, bbox_data=None, ego_data=None,
                temporal_data=None, cfg_scale: float = 1.0,
                return_cross_attention_contexts: bool = True) -> Dict[str, Any]:
        B, dev = self._batch_device(camera_data, road_data, bbox_data, ego_data, temporal_data)
        D = self.config.cond_dim
        embs, masks = [], []
        road_ctx = obj_tok = None
        for i, (name, data) in enumerate(zip(self.MODALITIES, (camera_data, road_data, bbox_data,
                                                              ego_data, temporal_data))):
            if not data:
                embs.append(self.null_tokens[i].expand(B, D))
                masks.append(torch.zeros(B, dtype=torch.bool, device=dev))
                continue
            if name == "camera":
                e = self.camera_encoder(data["intrinsics"], data["extrinsics"], data.get("camera_ids"))
            elif name == "road":
                e, road_ctx = self.road_encoder(data["waypoints"], data["road_type"], data["lane_info"],
                                                data.get("turn_info"), data.get("waypoint_mask"))
            elif name == "bbox":
                e, obj_tok = self.bbox_encoder(data["positions"], data["dimensions"], data["headings"],
                                               data["velocities"], data["object_classes"],
                                               data["confidences"], data.get("object_mask"))
            elif name == "ego":
                e = self.ego_encoder(data["position"], data["velocity"], data["acceleration"],
                                     data["heading"], data["heading_rate"], data.get("gps"), data.get("imu"))
            else:
                e = self.temporal_encoder(data["time_of_day"], data["weather"], data.get("weather_intensity"),
                                          data.get("season"), data.get("sun_azimuth"),
                                          data.get("sun_elevation"), data.get("lighting"))
            e, keep = self._apply_cfg_dropout(e, i)
            embs.append(e)
            masks.append(keep)
        cond = self.norm(self.fusion(torch.cat(embs, -1)))
        out = {"conditioning": cond, "adaln_params": self.adaln(cond),
               "modality_mask": torch.stack(masks, -1)}
        if return_cross_attention_contexts:
            out["road_context"] = None if road_ctx is None else self.context_proj(road_ctx)
            out["object_tokens"] = None if obj_tok is None else self.context_proj(obj_tok)
        return out

    def get_null_conditioning(self, batch_size: int, device) -> Dict[str, Any]:
        D = self.config.cond_dim
        embs = [self.null_tokens[i].expand(batch_size, D).to(device) for i in range(len(self.MODALITIES))]
        cond = self.norm(self.fusion(torch.cat(embs, -1)))
        return {"conditioning": cond, "adaln_params": self.adaln(cond)}

    @staticmethod
    def apply_cfg(cond_out: torch.Tensor, uncond_out: torch.Tensor, cfg_scale: float) -> torch.Tensor:
        return uncond_out + cfg_scale * (cond_out - uncond_out)


def create_conditioning_module(model_dim: int = 512, cond_dim: int = 256, num_cameras: int = 6,
                               max_waypoints: int = 50, max_objects: int = 64,
                               cfg_dropout_prob: float = 0.1, dropout: float = 0.1,
                               **kw) -> ConditioningIntegration:
    """(models/conditioning.py:1447-1475); other :class:`ConditioningConfig` fields by keyword."""
    return ConditioningIntegration(ConditioningConfig(
        model_dim=model_dim, cond_dim=cond_dim, num_cameras=num_cameras, max_waypoints=max_waypoints,
        max_objects=max_objects, cfg_dropout_prob=cfg_dropout_prob, dropout=dropout, **kw))
