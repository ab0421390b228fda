"""Restatement of the reference tensor environment's step math -- TEST
INFRASTRUCTURE ONLY (the checker of the fused env kernels; the product never
imports it).

Follows ``python/duck_gym/tensor_env.py`` of the reference: frame transforms
(:9-23, 221-236), observations (:238-258), termination, reward and time-outs
(:279-361).  The functions take the physics state read right after the
physics step and the env buffers, and return what the reference's ``step``
computes before its auto-reset.  Torch ops are kept in the reference's order
so that, on the same inputs, CPU results equal the reference's bit for bit
(pinned by ``tests/golden/env_*.npz``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def multiply(a, b):   # tensor_env.py:9-18
    return torch.cat(
        (
            a[..., :1] * b[..., :1] - (a[..., 1:] * b[..., 1:]).sum(-1, keepdim=True),
            a[..., :1] * b[..., 1:] + b[..., :1] * a[..., 1:] + torch.linalg.cross(a[..., 1:], b[..., 1:]),
        ),
        dim=-1,
    )


def inverse_rotate(q, v):   # tensor_env.py:21-23
    t = 2 * torch.linalg.cross(-q[..., 1:], v)
    return v + q[..., :1] * t + torch.linalg.cross(-q[..., 1:], t)


@dataclass
class EnvConfig:
    """The TensorEnv settings the step math reads."""

    task: str
    home: torch.Tensor          # [J]
    root_height: float
    root_iquat: list            # principal-frame quaternion of the root (wxyz)
    control_dt: float
    max_episode_length: int
    velocity_filter_seconds: float = 0.0
    velocity_alpha: float = 1.0
    tracking_weight: float = 4.0
    heading_weight: float = 0.4
    tracking_sigma: float = 0.04
    gait_period: float = 0.8
    tilt: float | None = None   # -cos(0.5) as the env's device computes it; None: this CPU's
    # Gait shaping (tensor_env.py:152-171, 263-277, 318-344), from gait.npz.
    gait: bool = False
    foot_clearance: bool = False
    load_transfer: bool = False
    gait_table: torch.Tensor | None = None     # [4, samples, J]
    gait_lift: float = 0.008
    foot_points: torch.Tensor | None = None    # [2, P, 3]
    foot_bodies: list | None = None
    mass: float = 0.0

    @property
    def iquat(self):   # tensor_env.py:137-139
        return torch.tensor(self.root_iquat, dtype=self.home.dtype) * torch.tensor([1, -1, -1, -1])


def reference_targets(episode_length, commands, cfg: EnvConfig):
    """tensor_env.py:263-277: HOME, or the gait table interpolated at the
    episode phase in the command's direction, blended in over the first
    second."""
    n = episode_length.shape[0]
    if not cfg.gait:
        return cfg.home.expand(n, -1)
    dt = cfg.home.dtype
    directions = torch.tensor([[1.0, 0], [-1, 0], [0, 1], [0, -1]], dtype=dt)
    phase = episode_length.to(dt) * cfg.control_dt / cfg.gait_period
    count = cfg.gait_table.shape[1]
    index = (phase % 1) * count
    lo = index.long()
    fraction = (index - lo)[:, None]
    direction = (commands @ directions.T).argmax(-1)
    ref = cfg.gait_table[direction, lo] * (1 - fraction) + cfg.gait_table[direction, (lo + 1) % count] * fraction
    blend = (episode_length.to(dt) * cfg.control_dt).clamp(0, 1)[:, None]
    return cfg.home + (ref - cfg.home) * blend


def features(b, cfg: EnvConfig):
    """tensor_env.py:221-236: body-frame gravity, velocities and heading."""
    n = b.shape[0]
    q = multiply(b[:, 1, 3:7], cfg.iquat.expand(n, -1))
    gravity = inverse_rotate(q, torch.tensor([0.0, 0, -1], dtype=b.dtype).expand(n, -1))
    v = inverse_rotate(q, b[:, 1, 7:10])
    w = inverse_rotate(q, b[:, 1, 10:13])
    yaw = torch.stack((1 - 2 * (q[:, 2] ** 2 + q[:, 3] ** 2), 2 * (q[:, 0] * q[:, 3] + q[:, 1] * q[:, 2])), dim=-1)
    return gravity, v, w, yaw


def observations(b, j, g, v, w, yaw, actions, episode_length, commands, filtered, cfg: EnvConfig):
    """tensor_env.py:238-258."""
    pieces = [g, v, w, b[:, 1, 2:3] - cfg.root_height, j[:, :, 0] - cfg.home, 0.1 * j[:, :, 1], actions]
    if cfg.task == "locomotion":
        phase = episode_length.to(b.dtype) * cfg.control_dt * (2 * torch.pi / cfg.gait_period)
        pieces.extend([commands, yaw, torch.stack((phase.sin(), phase.cos()), dim=-1)])
    if cfg.velocity_filter_seconds > 0:
        pieces.append(filtered)
    return torch.cat(pieces, dim=-1).float()


def post_step(b, j, d, a, prev_actions, episode_length, returns, commands, filtered, cfg: EnvConfig,
              contact_forces=None):
    """tensor_env.py:291-361: everything ``step`` computes after the physics
    and before its auto-reset.  Returns a dict with obs (the terminal
    observation), reward, failed, timeout, done and the updated buffers.
    ``contact_forces`` [E,B,3] (all contacts) feeds the load-transfer term."""
    g, v, w, yaw = features(b, cfg)
    height = b[:, 1, 2] - cfg.root_height
    tilt = -torch.cos(torch.tensor(0.5)) if cfg.tilt is None else torch.tensor(cfg.tilt)
    failed = ((g[:, 2] > tilt) | (height.abs() > 0.04) | (d[:, 0] > 0.005)
              | (d[:, 1] > 0.005) | (d[:, 5] > 0) | ~torch.isfinite(b).all(dim=(1, 2)))
    reward = (1.5 * torch.exp(-20 * g[:, :2].square().sum(-1)) + torch.exp(-2000 * height.square())
              + 0.5 * torch.exp(-10 * v.square().sum(-1)) - 0.02 * w.square().sum(-1)
              - 0.05 * (j[:, :, 0] - cfg.home).square().sum(-1) - 0.01 * a.square().sum(-1)
              - 0.02 * (a - prev_actions).square().sum(-1))
    filtered = filtered.clone()
    if cfg.task == "locomotion":
        velocity = b[:, 1, 7:9]
        if cfg.velocity_filter_seconds > 0:
            alpha = cfg.velocity_alpha
            filtered = (1 - alpha) * filtered + alpha * velocity
            velocity = filtered
        error = (velocity - commands).square().sum(-1)
        reward = (1.0 * torch.exp(-20 * g[:, :2].square().sum(-1)) + torch.exp(-2000 * height.square())
                  + cfg.tracking_weight * torch.exp(-error / cfg.tracking_sigma ** 2)
                  - 0.1 * w.square().sum(-1) - cfg.heading_weight * (1 - yaw[:, 0])
                  - 0.02 * a.square().sum(-1) - 0.03 * (a - prev_actions).square().sum(-1))
    if cfg.foot_clearance:   # tensor_env.py:318-333
        poses = b[:, cfg.foot_bodies]
        up = torch.tensor([0.0, 0, 1.0], dtype=b.dtype).expand(b.shape[0], 2, -1)
        local_up = inverse_rotate(poses[:, :, 3:7], up)
        heights = torch.einsum("fvi,efi->efv", cfg.foot_points, local_up) + poses[:, :, None, 2]
        clearance = heights.amin(-1)
        phase = ((episode_length[:, None] + 1) * cfg.control_dt / cfg.gait_period + torch.tensor([0.0, 0.5])) % 1
        swing = ((phase - 0.6) / 0.4).clamp(0, 1)
        desired = cfg.gait_lift * torch.sin(torch.pi * swing).square()
        reward -= 20000 * (clearance.clamp_min(0) - desired).square().sum(-1)
    if cfg.load_transfer:    # tensor_env.py:334-344
        forces = contact_forces[:, cfg.foot_bodies, 2].to(b.dtype) / (cfg.mass * 9.81)
        cycle = (episode_length.to(b.dtype) + 1) * cfg.control_dt / cfg.gait_period
        left = 0.5 + 0.5 * torch.sin(2 * torch.pi * (cycle - 0.05))
        wanted = torch.stack((left, 1 - left), dim=-1)
        reward -= 3 * (forces.clamp(0, 3) - wanted).square().sum(-1)
    reward = torch.where(failed, -2.0, reward) * cfg.control_dt
    episode_length = episode_length + 1
    returns = returns + reward.float()
    timeout = (episode_length >= cfg.max_episode_length) & ~failed
    done = failed | timeout
    obs = observations(b, j, g, v, w, yaw, a, episode_length, commands, filtered, cfg)
    return dict(obs=obs, reward=reward.float(), failed=failed, timeout=timeout, done=done,
                episode_length=episode_length, returns=returns, filtered=filtered, actions=a)


def config_from_fixture(config: dict, metadata: dict, dtype=torch.float32, gait_record=None) -> EnvConfig:
    cfg = EnvConfig(
        task=config["task"], home=torch.tensor(metadata["home"], dtype=dtype), root_height=metadata["root_height"],
        root_iquat=metadata["root_iquat"], control_dt=config["control_dt"],
        max_episode_length=config["max_episode_length"], velocity_filter_seconds=config["velocity_filter_seconds"],
        velocity_alpha=config["velocity_alpha"], tracking_weight=config["tracking_weight"],
        heading_weight=config["heading_weight"], tracking_sigma=config["tracking_sigma"])
    if config.get("gait"):
        apply_gait(cfg, gait_record, metadata, True, True, True)
    return cfg


def apply_gait(cfg: EnvConfig, record, metadata, gait, foot_clearance, load_transfer):
    """tensor_env.py:152-171: the gait.npz fields the shaping reads."""
    dt = cfg.home.dtype
    cfg.gait, cfg.foot_clearance, cfg.load_transfer = gait, foot_clearance, load_transfer
    cfg.gait_table = torch.tensor(record["targets"], dtype=dt)
    cfg.gait_period = float(record["period"])
    cfg.gait_lift = float(record["lift"]) if "lift" in record else 0.008
    cfg.foot_points = torch.tensor(record["foot_collision_points"], dtype=dt)
    cfg.foot_bodies = [int(v) for v in record["foot_bodies"]]
    cfg.mass = float(metadata["mass"])
    return cfg


__all__ = ["EnvConfig", "features", "observations", "post_step", "multiply", "inverse_rotate", "config_from_fixture",
           "math"]
