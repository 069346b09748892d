"""Closed-loop evaluation: observe -> plan -> act -> observe with the world model as the
simulator of observations.

API of the reference ``evaluation/closed_loop.py``: ``TaskType`` / ``TaskDefinition`` /
``EvaluationConfig`` / ``EvaluationResult`` (:26-206), ``ClosedLoopEvaluator``
(``evaluate_episode`` :278-375, ``evaluate_batch`` :377-414,
``evaluate_with_inference_scaling`` :416-458, sampling-based planning :498-646, kinematic
state update at 10 Hz :723-787, physics checks :849-870, result metrics :875-1197) and
the task factories (:1199-1240).

The world model here is a :class:`~drivedit_b200.models.world_dit.WorldDiT`:
observations are latent frames ``[C, H, W]``, each executed action produces the next
frame by a KV-cached Euler flow rollout (one frame per step, rolling window), exactly
the inference path. Planning samples ``num_trajectory_samples`` smooth action sequences
around the current plan and scores them with the kinematic model against the task
(goal distance, lateral deviation, comfort); ``num_planning_iterations`` refines the
best candidates (inference-time compute scaling).
"""
from __future__ import annotations

import math
import time
from collections import defaultdict
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional, Tuple

import torch


class TaskType(Enum):
    LANE_FOLLOWING = "lane_following"
    OBSTACLE_AVOIDANCE = "obstacle_avoidance"
    LANE_CHANGE = "lane_change"
    JUNCTION_NAVIGATION = "junction_navigation"
    PARKING = "parking"
    EMERGENCY_STOP = "emergency_stop"
    MERGE = "merge"
    ROUNDABOUT = "roundabout"
    PEDESTRIAN_CROSSING = "pedestrian_crossing"
    OPEN_ROAD = "open_road"


@dataclass
class TaskDefinition:
    task_type: TaskType
    name: str
    description: str = ""
    max_duration_steps: int = 300
    min_duration_steps: int = 10
    success_distance_threshold: float = 2.0
    max_lateral_deviation: float = 1.5
    max_heading_deviation: float = 0.5
    min_ttc: float = 2.0
    max_deceleration: float = 8.0
    max_jerk: float = 10.0
    goal_position: Optional[Tuple[float, float]] = None
    goal_heading: Optional[float] = None
    goal_speed: Optional[float] = None
    target_lane: Optional[int] = None
    weights: Dict[str, float] = field(default_factory=lambda: {
        "task_success": 0.4, "trajectory_quality": 0.2, "safety": 0.2, "comfort": 0.1, "efficiency": 0.1})

    def __post_init__(self):
        if self.task_type == TaskType.LANE_FOLLOWING:
            self.max_lateral_deviation = 0.5
        elif self.task_type == TaskType.EMERGENCY_STOP:
            self.max_deceleration = 10.0
            self.min_duration_steps = 5
        elif self.task_type == TaskType.JUNCTION_NAVIGATION:
            self.max_duration_steps = 500
        elif self.task_type == TaskType.PARKING:
            self.success_distance_threshold = 0.5
            self.max_heading_deviation = 0.1


@dataclass
class EvaluationConfig:
    num_planning_iterations: int = 1
    planning_horizon: int = 16
    replan_frequency: int = 4
    num_trajectory_samples: int = 8
    temperature: float = 0.8
    top_k: int = 5
    max_episode_steps: int = 1000
    context_length: int = 8
    prediction_horizon: int = 32
    enable_action_observation_scaling: bool = True
    action_observation_budget: int = 100
    enable_physics_checks: bool = True
    physics_violation_threshold: float = 0.1
    compute_detailed_metrics: bool = True
    log_frequency: int = 10
    flow_steps: int = 4
    window_frames: int = 32
    dt: float = 0.1


@dataclass
class EvaluationResult:
    task_success: bool
    task_completion_ratio: float
    success_rate: float
    trajectory_controllability: float
    action_response_alignment: float
    control_fidelity: float
    physics_violation_count: int
    physics_violation_ratio: float
    violation_details: Dict[str, int]
    average_displacement_error: float
    final_displacement_error: float
    trajectory_drift: float
    lateral_deviation_mean: float
    lateral_deviation_max: float
    collision_count: int
    near_miss_count: int
    min_time_to_collision: float
    safety_score: float
    max_acceleration: float
    max_jerk: float
    comfort_score: float
    task_duration_steps: int
    path_efficiency: float
    speed_efficiency: float
    planning_iterations_used: int
    avg_inference_time_ms: float
    total_evaluation_time_s: float
    predictions: Optional[torch.Tensor] = None
    ground_truth: Optional[torch.Tensor] = None
    actions_taken: Optional[torch.Tensor] = None

    def to_dict(self) -> Dict[str, Any]:
        d = asdict(self)
        for k in ("predictions", "ground_truth", "actions_taken"):
            d.pop(k, None)
        return d


def kinematic_step(state: Dict[str, torch.Tensor], action: torch.Tensor, dt: float) -> Dict[str, torch.Tensor]:
    """Unicycle update: ``action = [steering (yaw rate, rad/s), acceleration (m/s^2),
    ...]``; batched over leading dims of ``action``."""
    steer, acc = action[..., 0], action[..., 1]
    speed = (state["speed"] + acc * dt).clamp_min(0.0)
    heading = state["heading"] + steer * dt
    vel = torch.stack([speed * torch.cos(heading), speed * torch.sin(heading)], -1)
    return {"position": state["position"] + vel * dt, "velocity": vel, "heading": heading, "speed": speed,
            "acceleration": acc, "steering": steer}


class ClosedLoopEvaluator:
    def __init__(self, world_model, config: EvaluationConfig, physics_detector=None, driving_metrics=None,
                 device: str = "cuda"):
        self.world_model = world_model
        self.config = config
        self.physics_detector, self.driving_metrics = physics_detector, driving_metrics
        self.device = torch.device(device if (device != "cuda" or torch.cuda.is_available()) else "cpu")
        self.world_model.to(self.device).eval()
        self.dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.A = world_model.cfg.action_dim
        self.gen = torch.Generator(device="cpu").manual_seed(0)
        self.reset()

    def reset(self) -> None:
        self.episode_step = 0
        self.context_buffer: List[torch.Tensor] = []
        self.action_buffer: List[torch.Tensor] = []
        self.state_buffer: List[Dict[str, torch.Tensor]] = []
        self.predictions_history: List[torch.Tensor] = []
        self.ground_truth_history: List[torch.Tensor] = []
        self.actions_history: List[torch.Tensor] = []
        self.inference_times: List[float] = []
        self.violation_counts: Dict[str, int] = defaultdict(int)
        self.plan: Optional[torch.Tensor] = None
        self.cache = None
        self.planning_iterations = 0

    # ------------------------------------------------------------------ model io
    def _initialize_context(self, initial_observation: torch.Tensor) -> None:
        from ..models.world_dit import KVCacheSet, forward_cached

        obs = initial_observation.to(self.device, self.dtype)
        if obs.dim() == 3:
            obs = obs[None]
        self.cache = KVCacheSet(self.world_model, 1, self.config.window_frames, 1, self.device, self.dtype)
        a = torch.zeros(1, obs.shape[0], self.A, device=self.device)
        with torch.no_grad():
            forward_cached(self.world_model, obs[None], torch.ones(1, device=self.device), a, self.cache, commit=True)
        self.context_buffer.extend(list(obs))

    def _get_current_observation(self) -> torch.Tensor:
        return torch.stack(self.context_buffer[-self.config.context_length:])

    @torch.no_grad()
    def _predict_next(self, action: torch.Tensor) -> torch.Tensor:
        from ..models.world_dit import forward_cached

        m = self.world_model
        shape = (1, 1) + tuple(self.context_buffer[-1].shape)
        x = torch.randn(shape, generator=self.gen).to(self.device, self.dtype)
        a = action.view(1, 1, -1)[..., :self.A].to(self.device).float()
        ts = torch.linspace(0, 1, self.config.flow_steps + 1)
        for i in range(self.config.flow_steps):
            v = forward_cached(m, x, ts[i].expand(1).to(self.device), a, self.cache, commit=False)
            x = (x.float() + float(ts[i + 1] - ts[i]) * v.float()).to(self.dtype)
        forward_cached(m, x, torch.ones(1, device=self.device), a, self.cache, commit=True)
        return x[0, 0]

    # ------------------------------------------------------------------ planning
    def _sample_actions(self, n: int, horizon: int) -> torch.Tensor:
        base = self.plan if self.plan is not None else torch.zeros(horizon, self.A)
        if base.shape[0] < horizon:
            base = torch.cat([base, base[-1:].expand(horizon - base.shape[0], -1)], 0)
        noise = torch.randn(n, horizon, self.A, generator=self.gen) * self.config.temperature * 0.5
        k = torch.tensor([0.25, 0.5, 0.25])  # temporal smoothing of the perturbations
        noise = torch.nn.functional.conv1d(noise.transpose(1, 2).reshape(-1, 1, horizon),
                                           k.view(1, 1, 3), padding=1).view(n, self.A, horizon).transpose(1, 2)
        cand = (base[None, :horizon] + noise).clamp(-1, 1)
        cand[0] = base[:horizon].clamp(-1, 1)
        # motion primitives: constant acceleration levels, straight steering
        prim = torch.zeros(5, horizon, self.A)
        prim[:, :, 1] = torch.tensor([-1.0, -0.5, 0.0, 0.5, 1.0])[:, None]
        return torch.cat([cand, prim], 0)

    def _evaluate_trajectory(self, actions: torch.Tensor, task: TaskDefinition) -> torch.Tensor:
        """Kinematic cost of ``[N, H, A]`` candidate sequences from the current state."""
        st = self.state_buffer[-1]
        s = {k: v.expand(actions.shape[0], *v.shape) for k, v in st.items()}
        cost = torch.zeros(actions.shape[0])
        prev_acc = s["acceleration"]
        for h in range(actions.shape[1]):
            s = kinematic_step(s, actions[:, h] * torch.tensor([0.5, 4.0] + [1.0] * (self.A - 2)), self.config.dt)
            jerk = (s["acceleration"] - prev_acc).abs() / self.config.dt
            prev_acc = s["acceleration"]
            cost += 0.002 * jerk + 0.1 * s["position"][:, 1].abs()
            if task.goal_speed is not None:
                cost += 0.5 * (s["speed"] - task.goal_speed).abs()
        if task.goal_position is not None:
            cost += (s["position"] - torch.tensor(task.goal_position)).norm(dim=-1)
        return cost

    def _predict_with_planning(self, task: TaskDefinition) -> torch.Tensor:
        c = self.config
        best = None
        for _ in range(max(1, c.num_planning_iterations)):
            cand = self._sample_actions(c.num_trajectory_samples, c.planning_horizon)
            cost = self._evaluate_trajectory(cand, task)
            top = cost.topk(min(c.top_k, len(cost)), largest=False).indices
            best = cand[top[0]]
            self.plan = cand[top].mean(0)  # refine around the elite set
            self.planning_iterations += 1
        self.plan = best
        return best

    def _select_action(self, task: TaskDefinition) -> torch.Tensor:
        if self.plan is None or self.episode_step % self.config.replan_frequency == 0:
            self._predict_with_planning(task)
        a = self.plan[0]
        self.plan = torch.cat([self.plan[1:], self.plan[-1:]], 0)
        return a

    # ------------------------------------------------------------------ env step
    def _simulate_step(self, action: torch.Tensor) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
        t0 = time.perf_counter()
        obs = self._predict_next(action)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.inference_times.append((time.perf_counter() - t0) * 1000.0)
        scaled = action * torch.tensor([0.5, 4.0] + [1.0] * (self.A - 2))
        return obs, kinematic_step(self.state_buffer[-1], scaled, self.config.dt)

    def _update_context(self, observation, state_info, action) -> None:
        self.context_buffer.append(observation)
        self.state_buffer.append(state_info)
        self.action_buffer.append(action)
        keep = max(self.config.context_length, 2)
        if len(self.context_buffer) > keep:
            self.context_buffer = self.context_buffer[-keep:]

    def _check_task_complete(self, task: TaskDefinition) -> bool:
        st = self.state_buffer[-1]
        if task.task_type == TaskType.EMERGENCY_STOP:
            return float(st["speed"]) < 0.1 and self.episode_step >= task.min_duration_steps
        if task.goal_position is not None:
            d = float((st["position"] - torch.tensor(task.goal_position)).norm())
            return d < task.success_distance_threshold
        return self.episode_step >= task.max_duration_steps

    def _check_collision(self) -> bool:
        return False  # no obstacle map without an environment

    def _check_physics_violations(self, state_info: Dict[str, torch.Tensor], task: TaskDefinition) -> None:
        if len(self.state_buffer) >= 2:
            if float(state_info["acceleration"]) < -task.max_deceleration:
                self.violation_counts["max_deceleration"] += 1
            jerk = abs(float(state_info["acceleration"] - self.state_buffer[-1]["acceleration"])) / self.config.dt
            if jerk > task.max_jerk:
                self.violation_counts["max_jerk"] += 1
        if float(state_info["speed"]) > 60.0:
            self.violation_counts["speed_limit"] += 1

    def _trigger_replan(self) -> None:
        self.plan = None

    # ------------------------------------------------------------------ episodes
    def evaluate_episode(self, task: TaskDefinition, initial_observation: torch.Tensor,
                         initial_state: Dict[str, torch.Tensor], environment=None,
                         ground_truth_trajectory: Optional[torch.Tensor] = None) -> EvaluationResult:
        t_start = time.perf_counter()
        self.reset()
        self._initialize_context(initial_observation)
        st = {"position": torch.as_tensor(initial_state.get("position", torch.zeros(2)), dtype=torch.float32),
              "heading": torch.as_tensor(initial_state.get("heading", 0.0), dtype=torch.float32).reshape(()),
              "speed": torch.as_tensor(initial_state.get("speed", 5.0), dtype=torch.float32).reshape(()),
              "acceleration": torch.zeros(()), "steering": torch.zeros(())}
        st["velocity"] = torch.stack([st["speed"] * torch.cos(st["heading"]), st["speed"] * torch.sin(st["heading"])])
        self.state_buffer.append(st)
        success = False
        steps = min(task.max_duration_steps, self.config.max_episode_steps)
        for _ in range(steps):
            action = self._select_action(task)
            if environment is not None:
                obs, info = environment.step(action)
            else:
                obs, info = self._simulate_step(action)
            if self.config.enable_physics_checks:
                self._check_physics_violations(info, task)
            self._update_context(obs, info, action)
            self.actions_history.append(action)
            self.predictions_history.append(info["position"])
            self.episode_step += 1
            if self._check_collision():
                self._trigger_replan()
            if self._check_task_complete(task):
                success = True
                break
        return self._compute_evaluation_result(task, success, ground_truth_trajectory,
                                               time.perf_counter() - t_start)

    def evaluate_batch(self, tasks: List[TaskDefinition], initial_observations, initial_states,
                       environments=None) -> Dict[str, Any]:
        res = [self.evaluate_episode(t, o, s, None if environments is None else environments[i])
               for i, (t, o, s) in enumerate(zip(tasks, initial_observations, initial_states))]
        sr = sum(r.task_success for r in res) / max(len(res), 1)
        for r in res:
            r.success_rate = sr
        return {"results": res, "success_rate": sr,
                "mean_ade": sum(r.average_displacement_error for r in res) / max(len(res), 1),
                "mean_inference_ms": sum(r.avg_inference_time_ms for r in res) / max(len(res), 1)}

    def evaluate_with_inference_scaling(self, task, initial_observation, initial_state,
                                        planning_iterations=(1, 2, 4)) -> Dict[int, EvaluationResult]:
        out = {}
        base = self.config.num_planning_iterations
        for n in planning_iterations:
            self.config.num_planning_iterations = n
            out[n] = self.evaluate_episode(task, initial_observation, initial_state)
        self.config.num_planning_iterations = base
        return out

    # ------------------------------------------------------------------ metrics
    def _positions(self) -> torch.Tensor:
        return torch.stack([s["position"] for s in self.state_buffer])

    def _compute_trajectory_metrics(self, gt: Optional[torch.Tensor]) -> Tuple[float, float, float]:
        pos = self._positions()
        if gt is None or gt.shape[0] < 2:
            drift = float((pos[-1] - pos[0]).norm()) if len(pos) > 1 else 0.0
            return 0.0, 0.0, drift
        n = min(len(pos), gt.shape[0])
        err = (pos[:n] - gt[:n, :2].float()).norm(dim=-1)
        return float(err.mean()), float(err[-1]), float(err.max())

    def _compute_lateral_deviation(self) -> Tuple[float, float]:
        lat = self._positions()[:, 1].abs()
        return float(lat.mean()), float(lat.max())

    def _compute_comfort_metrics(self) -> Tuple[float, float]:
        acc = torch.stack([s["acceleration"] for s in self.state_buffer])
        jerk = (acc[1:] - acc[:-1]).abs() / self.config.dt if len(acc) > 1 else torch.zeros(1)
        return float(acc.abs().max()), float(jerk.max())

    @staticmethod
    def _compute_comfort_score(max_acc: float, max_jerk: float, task: TaskDefinition) -> float:
        return max(0.0, 1.0 - 0.5 * max_acc / task.max_deceleration - 0.5 * max_jerk / task.max_jerk)

    def _compute_path_efficiency(self) -> float:
        pos = self._positions()
        if len(pos) < 2:
            return 1.0
        path = (pos[1:] - pos[:-1]).norm(dim=-1).sum()
        return float((pos[-1] - pos[0]).norm() / path.clamp_min(1e-6))

    def _compute_speed_efficiency(self, task: TaskDefinition) -> float:
        sp = torch.stack([s["speed"] for s in self.state_buffer])
        if task.goal_speed is None:
            return 1.0
        return float(1.0 - ((sp - task.goal_speed).abs() / max(task.goal_speed, 1e-6)).clamp(0, 1).mean())

    def _compute_controllability(self) -> float:
        """Share of steps where the heading change has the sign of the steering command."""
        if len(self.state_buffer) < 2:
            return 1.0
        steer = torch.stack([a[0] for a in self.actions_history])
        dh = torch.stack([s["heading"] for s in self.state_buffer])
        dh = dh[1:] - dh[:-1]
        n = min(len(steer), len(dh))
        agree = ((torch.sign(steer[:n]) == torch.sign(dh[:n])) | (steer[:n].abs() < 1e-3)).float()
        return float(agree.mean())

    def _compute_action_response_alignment(self) -> float:
        """Correlation between commanded and realised acceleration."""
        if len(self.actions_history) < 3:
            return 1.0
        a = torch.stack([x[1] for x in self.actions_history]).float()
        r = torch.stack([s["acceleration"] for s in self.state_buffer[1:]]).float()
        a, r = a - a.mean(), r - r.mean()
        return float((a * r).sum() / (a.norm() * r.norm()).clamp_min(1e-9))

    def _compute_control_fidelity(self) -> float:
        """How much consecutive predicted latent frames respond to the action change."""
        if len(self.context_buffer) < 3:
            return 1.0
        f = torch.stack(self.context_buffer[-3:]).float()
        return float(1.0 / (1.0 + (f[2] - 2 * f[1] + f[0]).pow(2).mean()))

    def _compute_evaluation_result(self, task, success, gt, elapsed) -> EvaluationResult:
        ade, fde, drift = self._compute_trajectory_metrics(gt)
        lat_mean, lat_max = self._compute_lateral_deviation()
        max_acc, max_jerk = self._compute_comfort_metrics()
        nviol = sum(self.violation_counts.values())
        steps = max(self.episode_step, 1)
        return EvaluationResult(
            task_success=success, task_completion_ratio=1.0 if success else self.episode_step / max(task.max_duration_steps, 1),
            success_rate=float(success), trajectory_controllability=self._compute_controllability(),
            action_response_alignment=self._compute_action_response_alignment(),
            control_fidelity=self._compute_control_fidelity(), physics_violation_count=nviol,
            physics_violation_ratio=nviol / steps, violation_details=dict(self.violation_counts),
            average_displacement_error=ade, final_displacement_error=fde, trajectory_drift=drift,
            lateral_deviation_mean=lat_mean, lateral_deviation_max=lat_max, collision_count=0, near_miss_count=0,
            min_time_to_collision=float("inf"), safety_score=max(0.0, 1.0 - nviol / steps),
            max_acceleration=max_acc, max_jerk=max_jerk,
            comfort_score=self._compute_comfort_score(max_acc, max_jerk, task), task_duration_steps=self.episode_step,
            path_efficiency=self._compute_path_efficiency(), speed_efficiency=self._compute_speed_efficiency(task),
            planning_iterations_used=self.planning_iterations,
            avg_inference_time_ms=sum(self.inference_times) / max(len(self.inference_times), 1),
            total_evaluation_time_s=elapsed, predictions=self._positions(), ground_truth=gt,
            actions_taken=torch.stack(self.actions_history) if self.actions_history else None)


def create_lane_following_task(name: str = "lane_following", max_duration: int = 300,
                               target_speed: float = 10.0) -> TaskDefinition:
    """Keep the lane at ``target_speed`` for up to ``max_duration`` steps
    (evaluation/closed_loop.py:1199-1211)."""
    return TaskDefinition(TaskType.LANE_FOLLOWING, name, "keep the lane at a safe constant speed",
                          max_duration_steps=max_duration, max_lateral_deviation=0.5,
                          goal_speed=target_speed)


def create_obstacle_avoidance_task(obstacle_position=(20.0, 0.0), name: str = "obstacle_avoidance",
                                   max_duration: int = 200) -> TaskDefinition:
    """Pass an obstacle at ``obstacle_position`` (metres ahead, lateral) keeping a
    time-to-collision of at least 2 s; the goal is 10 m past it
    (evaluation/closed_loop.py:1214-1225)."""
    return TaskDefinition(TaskType.OBSTACLE_AVOIDANCE, name, "avoid the obstacle while making progress",
                          max_duration_steps=max_duration, min_ttc=2.0,
                          goal_position=(obstacle_position[0] + 10.0, obstacle_position[1]))


def create_emergency_stop_task(name: str = "emergency_stop", max_duration: int = 50) -> TaskDefinition:
    """Stop completely as fast as the deceleration limit allows
    (evaluation/closed_loop.py:1228-1240)."""
    return TaskDefinition(TaskType.EMERGENCY_STOP, name, "come to a complete stop quickly and safely",
                          max_duration_steps=max_duration, min_duration_steps=5,
                          max_deceleration=10.0, goal_speed=0.0)
