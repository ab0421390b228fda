"""Restatement of the reference BAM environment's step math -- TEST
INFRASTRUCTURE ONLY (the checker of the fused BAM kernels; the product never
imports it).

Follows the reference's ``python/duck_gym``:
  * ``actuator.py:16-77``      the XL330/m6 servo (BAM, third-party ``bam``
                               package at commit 62bd8ce, restated there);
  * ``bam_env.py:136-170``     ``refresh`` frames (gravity, body velocities,
                               foot contacts and sole sites);
  * ``bam_env.py:185-211``     actor / critic observations;
  * ``bam_env.py:292-389``     per-substep delay ring, servo, bookkeeping;
  * ``bam_env.py:409-447``     failure rule and reward features;
  * ``walking_reward.py:45-96`` reward terms and their weights.

Torch ops are kept in the reference's order so that, on the same inputs, CPU
results equal the reference's bit for bit (pinned by
``tests/golden/bam_*.npz``).  Every function takes the physics quantities as
arguments -- body states, joint states, generalized loads, contact forces --
so the checker runs on states read from any engine.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .env_math import inverse_rotate, multiply

CONJ = (1, -1, -1, -1)


def xl330_m6(target, position, velocity, previous_motor, previous_applied, external, p, *, vin, vin_drop_gain,
             vin_min, kp_fw, force_limit, kp_scale=1.0, kd_scale=1.0, friction_scale=1.0):
    """actuator.py:16-77: motor channels (applied torque, dry-friction budget,
    viscous damping) [E,J,3], raw torque [E,J] and supply voltage [E,1]."""
    supply = (vin - vin_drop_gain * previous_motor.abs().sum(-1, keepdim=True)).clamp(min=vin_min)
    speed = velocity * kd_scale
    kt, res = p["kt"], p["R"]
    counts_per_rad = (4096 / (2 * math.pi)) / (256 * 885)
    duty = (target - position) * kp_fw * kp_scale * counts_per_rad
    center = kt * speed / supply
    span = res * 1.75 / supply
    duty = duty.clamp(min=center - span, max=center + span).clamp(-1.0, 1.0)
    raw = kt * supply * duty / res - kt ** 2 * speed / res
    stribeck = torch.exp(-torch.pow(velocity.abs() / p["dtheta_stribeck"], p["alpha"]))
    mot, ext = previous_applied, external
    quad = torch.where(mot.abs() > ext.abs(), p["load_friction_external_quad"] * ext.square(),
                       p["load_friction_motor_quad"] * mot.square())
    budget = (p["friction_base"] + stribeck * p["friction_stribeck"]
              + (ext * p["load_friction_external"] - mot * p["load_friction_motor"]).abs()
              + stribeck * (ext * p["load_friction_external_stribeck"]
                            - mot * p["load_friction_motor_stribeck"]).abs()
              + stribeck * quad) * friction_scale
    applied = raw.clamp(min=-force_limit, max=force_limit)
    damping = torch.full_like(applied, p["friction_viscous"])
    return torch.stack((applied, budget, damping), dim=-1), raw, supply


@dataclass
class BamConfig:
    """The BamEnv settings the step math reads (from its config.json and
    training dictionary)."""

    home: torch.Tensor              # [E,J]
    root_offset: torch.Tensor       # [E,3]
    root_rotation_inv: torch.Tensor  # [4]
    foot_ids: list
    foot_sites: torch.Tensor        # [2,3]
    mass: torch.Tensor              # [B]
    inertia: torch.Tensor           # [B,3]
    soft_limits: torch.Tensor       # [E,J,2]
    joint_names: list
    dt: float
    step_dt: float
    max_episode_length: int
    mean_velocity_tau: float = 0.0
    heading_reward_weight: float = 0.0
    heading_hold: bool = False
    linear_variance: float = 0.1
    vertical_variance: float = 0.1
    training: dict | None = None
    reward_weight_overrides: dict = field(default_factory=dict)

    @property
    def head_ids(self):
        return [i for i, n in enumerate(self.joint_names) if "head" in n or "neck" in n]

    @property
    def leg_ids(self):
        return [i for i in range(len(self.joint_names)) if i not in self.head_ids]


def frames(bodies, contact_force, cfg: BamConfig):
    """bam_env.py:136-170 (contact_force: the ground-only contact forces of
    the feet, [E,2,3])."""
    n = bodies.shape[0]
    dev, dt = bodies.device, bodies.dtype
    sign = torch.tensor(CONJ, device=dev, dtype=dt)
    root_quat = multiply(bodies[:, 1, 3:7], cfg.root_rotation_inv.expand(n, -1))
    gravity = inverse_rotate(root_quat, torch.tensor([0.0, 0.0, -1.0], device=dev, dtype=dt).expand(n, -1))
    ang_vel = inverse_rotate(root_quat, bodies[:, 1, 10:13])
    root_r = -inverse_rotate(bodies[:, 1, 3:7] * sign, cfg.root_offset)
    origin_vel = bodies[:, 1, 7:10] + torch.linalg.cross(bodies[:, 1, 10:13], root_r)
    lin_vel = inverse_rotate(root_quat, origin_vel)
    contact = contact_force.norm(dim=-1) > 1e-5
    foot = bodies[:, cfg.foot_ids]
    conj = foot[:, :, 3:7] * sign
    r = inverse_rotate(conj, cfg.foot_sites[None, :, :].expand(n, -1, -1))
    return dict(root_quat=root_quat, gravity=gravity, ang_vel=ang_vel, origin_world_velocity=origin_vel,
                lin_vel=lin_vel, contact_force=contact_force, contact=contact,
                site_pos=foot[:, :, :3] + r, site_vel=foot[:, :, 7:10] + torch.linalg.cross(foot[:, :, 10:13], r))


def yaw(root_quat):
    q = root_quat
    return torch.atan2(2 * (q[:, 0] * q[:, 3] + q[:, 1] * q[:, 2]), 1 - 2 * (q[:, 2].square() + q[:, 3].square()))


def heading_error(target_yaw, root_quat):
    error = target_yaw - yaw(root_quat)
    return torch.atan2(error.sin(), error.cos())


def observations(f, joints, home, observed_velocity, action, command, mean_velocity_world=None,
                 heading=None):
    """bam_env.py:185-211: actor [E,61] and critic [E,76(+3)(+1)]."""
    n, dev, dt = joints.shape[0], joints.device, joints.dtype
    pad = torch.zeros(n, 10, device=dev, dtype=dt)
    actor = torch.cat((f["ang_vel"], f["gravity"], joints[:, :, 0] - home, observed_velocity, action, command, pad),
                      dim=-1).float()
    forces = f["contact_force"].flatten(1)
    critic = torch.cat((f["lin_vel"], f["ang_vel"], f["gravity"], joints[:, :, 0] - home, joints[:, :, 1], action,
                        command, f["site_pos"][:, :, 2], f["air_time"], f["contact"].to(dt),
                        forces.sign() * forces.abs().log1p(), pad), dim=-1).float()
    if mean_velocity_world is not None:
        critic = torch.cat((critic, inverse_rotate(f["root_quat"], mean_velocity_world).float()), dim=-1)
    if heading is not None:
        critic = torch.cat((critic, heading[:, None].float()), dim=-1)
    return {"actor": actor, "critic": critic}


def failure(gravity, diag, self_penetration, joints):
    """bam_env.py:409-418."""
    return ((gravity[:, 2] > -math.cos(math.radians(70.0))) | (diag[:, 5] > 0) | (diag[:, 0] > 0.005)
            | (diag[:, 1] > 0.005) | (self_penetration > 0.005) | (~torch.isfinite(joints).all(dim=(1, 2))))


def angular_momentum(bodies, cfg: BamConfig):
    """bam_env.py:419-428."""
    q = bodies[:, :, 3:7]
    sign = cfg.home.new_tensor(CONJ)
    local_w = inverse_rotate(q, bodies[:, :, 10:13])
    spin = inverse_rotate(q * sign, cfg.inertia[None, :, :] * local_w)
    com = (bodies[:, :, :3] * cfg.mass[None, :, None]).sum(1) / cfg.mass.sum()
    orbital = torch.linalg.cross(bodies[:, :, :3] - com[:, None, :], bodies[:, :, 7:10] * cfg.mass[None, :, None])
    return (spin + orbital).sum(1)


class WalkingTerms:
    """walking_reward.py:15-122 with its two pieces of state (swing peak
    heights and the head-pose moving average)."""

    GAINS = dict(hip_yaw=(0.1, 0.3), hip_roll=(0.05, 0.05), hip_pitch=(0.15, 0.4), knee=(0.15, 0.4),
                 ankle=(0.1, 0.25))

    def __init__(self, cfg: BamConfig):
        self.cfg = cfg
        home = cfg.home
        keys = [next(k for k in self.GAINS if k in cfg.joint_names[i]) for i in cfg.leg_ids]
        self.stand = home.new_tensor([self.GAINS[k][0] for k in keys])
        self.walk = home.new_tensor([self.GAINS[k][1] for k in keys])
        self.head_ema = torch.zeros_like(home[:, cfg.head_ids])
        self.peak_height = home.new_zeros((len(home), 2))

    def reset(self, mask):
        self.head_ema[mask] = 0
        self.peak_height[mask] = 0

    def terms(self, f, dt):
        cfg = self.cfg
        command = f["command"]
        speed = command[:, :2].norm(dim=-1) + command[:, 2].abs()
        active = (speed > 0.01).to(cfg.home.dtype)
        std = torch.where((speed < 0.01)[:, None], self.stand, self.walk)
        pose_error = f["joint_pos"] - cfg.home
        height = f["foot_height"]
        foot_speed2 = f["foot_vel"][:, :, :2].square().sum(-1)
        first = (f["contact_time"] > 0) & (f["contact_time"] < dt + 1e-8)
        self.peak_height = torch.where(~f["contact"], torch.maximum(self.peak_height, height), self.peak_height)
        swing_cost = ((self.peak_height / 0.02 - 1).square() * first).sum(-1) * active
        self.peak_height = torch.where(first, 0.0, self.peak_height)
        head_error = pose_error[:, cfg.head_ids] - f["head_command"]
        self.head_ema[f["episode_steps"] <= 1] = 0
        alpha = min(1.0, dt / 1.0)
        self.head_ema = (1 - alpha) * self.head_ema + alpha * head_error
        return {
            "track_linear_velocity": torch.exp(-(f["lin_vel"][:, :2] - command[:, :2]).square().sum(-1)
                                               / cfg.linear_variance
                                               - f["lin_vel"][:, 2].square() / cfg.vertical_variance),
            "track_angular_velocity": torch.exp(-((f["ang_vel"][:, 2] - command[:, 2]).square()
                                                  + f["ang_vel"][:, :2].square().sum(-1)) / 0.5),
            "upright": torch.exp(-f["gravity"][:, :2].square().sum(-1) / 0.05),
            "pose": torch.exp(-(pose_error[:, cfg.leg_ids] / std).square().mean(-1)),
            "body_ang_vel": f["world_ang_vel"][:, :2].square().sum(-1),
            "angular_momentum": f["angular_momentum"].square().sum(-1),
            "dof_pos_limits": ((cfg.soft_limits[:, :, 0] - f["joint_pos"]).clamp(min=0)
                               + (f["joint_pos"] - cfg.soft_limits[:, :, 1]).clamp(min=0)).sum(-1),
            "action_rate_l2": (f["action"] - f["previous_action"]).square().sum(-1),
            "air_time": ((f["air_time"] > 0.125) & (f["air_time"] < 0.3)).sum(-1) * active,
            "foot_clearance": ((height - 0.02).abs() * foot_speed2.sqrt()).sum(-1) * active,
            "foot_swing_height": swing_cost,
            "foot_slip": (foot_speed2 * f["contact"]).sum(-1) * active,
            "self_collisions": f["self_collisions"],
            "head_pose_tracking": torch.exp(-(head_error / 0.5).square()).mean(-1),
            "head_pose_bias": -self.head_ema.abs().mean(-1),
        }


def walking_weights(iteration):
    """walking_reward.py:98-122: the curriculum of the action-rate and
    head-bias weights; the other weights are constant."""
    action = -0.1
    for start, w in ((500, -0.2), (750, -0.4), (1000, -0.6), (1250, -0.8), (1500, -1.0)):
        if iteration >= start:
            action = w
    head = 0.0
    for start, w in ((600, 1.0), (1000, 2.0), (1500, 3.0)):
        if iteration >= start:
            head = w
    return dict(track_linear_velocity=2.0, track_angular_velocity=2.0, upright=2.0, pose=1.0, body_ang_vel=-0.05,
                angular_momentum=-0.02, dof_pos_limits=-1.0, action_rate_l2=action, air_time=3.0,
                foot_clearance=-2.0, foot_swing_height=-0.25, foot_slip=-0.1, self_collisions=-1.0,
                head_pose_tracking=2.0, head_pose_bias=head)


def soft_limits_from_model(model_text: str, num_envs: int, dtype=torch.float32):
    """bam_env.py:72-80: joint limits shrunk to 90 % about their centres."""
    lines = model_text.splitlines()
    body_count = int(lines[0].split()[2])
    rows = [line.split() for line in lines[2 + body_count:2 + body_count + 14]]
    limits = torch.tensor([[float(r[22]), float(r[23])] for r in rows], dtype=dtype)
    center = limits.mean(-1, keepdim=True)
    return (center + 0.9 * (limits - center))[None, :, :].expand(num_envs, -1, -1)


def body_table(model_text: str, dtype=torch.float32):
    """bam_env.py:72-76: body masses and principal inertias from the model."""
    lines = model_text.splitlines()
    body_count = int(lines[0].split()[2])
    rows = [line.split() for line in lines[2:2 + body_count]]
    return (torch.tensor([float(r[1]) for r in rows], dtype=dtype),
            torch.tensor([[float(v) for v in r[2:5]] for r in rows], dtype=dtype))


class BamStepper:
    """bam_env.py:292-389: one control step of the BAM environment over an
    abstract physics engine ``native`` with the reference CudaBatch methods
    (``generalized_loads``, ``step_motor``, ``state``, ``contact_forces``,
    ``self_contact_stats``) returning torch tensors.  The env buffers live in
    ``self.buf`` (names as in the reference BamEnv); ``step`` returns what the
    reference's ``step`` computes before its auto-reset."""

    BUFFERS = ("action", "old_action", "previous_motor", "previous_applied", "observed_velocity", "command",
               "mean_velocity_world", "target_yaw", "air_time", "contact_time", "episode_length_buf",
               "target_history", "history_initialized", "self_contacts", "self_penetration", "joints",
               "head_ema", "peak_height")

    def __init__(self, native, cfg: BamConfig, config_json: dict, lag: int, decimation: int, reward_enabled=True,
                 source_iteration=0, neutral_head=False, head_stability=None):
        self.native, self.cfg, self.json = native, cfg, config_json
        self.lag, self.decimation = lag, decimation
        self.reward_enabled, self.source_iteration = reward_enabled, source_iteration
        self.neutral_head, self.head_stability = neutral_head, head_stability or {}
        self.reward = WalkingTerms(cfg)
        self.buf = {}
        self.history_cursor = 0
        self.common_step_counter = 0

    def load(self, buffers: dict, history_cursor: int, common_step_counter: int):
        self.buf = {k: v.clone() for k, v in buffers.items()}
        self.reward.head_ema = self.buf.pop("head_ema")
        self.reward.peak_height = self.buf.pop("peak_height")
        self.history_cursor, self.common_step_counter = history_cursor, common_step_counter

    def _frames(self):
        b, j, d = self.native.state()
        foot_force = self.native.contact_forces(ground_only=True)[:, self.cfg.foot_ids]
        f = frames(b, foot_force, self.cfg)
        f.update(bodies=b, joints=j, diag=d)
        return f

    def step(self, actions):
        cfg, buf, js = self.cfg, self.buf, self.json
        buf["old_action"] = buf["action"].clone()
        buf["action"] = actions.to(cfg.home.dtype).clone()
        if self.neutral_head:
            buf["action"][:, cfg.head_ids] = 0
        buf["observed_velocity"] = buf["joints"][:, :, 1].clone()
        target = cfg.home + buf["action"]
        buf["self_contacts"] = torch.zeros_like(buf["self_contacts"])
        buf["self_penetration"] = torch.zeros_like(buf["self_penetration"])
        n = target.shape[0]
        hist = buf["target_history"]
        for _ in range(self.decimation):
            hist[self.history_cursor] = target
            new = ~buf["history_initialized"]
            hist[:, new] = target[new]
            buf["history_initialized"][:] = True
            delayed = hist[(self.history_cursor - self.lag) % (self.lag + 1)]
            self.history_cursor = (self.history_cursor + 1) % (self.lag + 1)
            loads = self.native.generalized_loads(cfg.root_offset)
            motor, raw, _ = xl330_m6(
                delayed, buf["joints"][:, :, 0], buf["joints"][:, :, 1], buf["previous_motor"],
                buf["previous_applied"], -loads[:, :, 0] + loads[:, :, 1], js["parameters"],
                vin=torch.full((n, 1), js["vin"], device=target.device, dtype=target.dtype),
                vin_drop_gain=js["vin_drop_gain"], vin_min=js["vin_min"], kp_fw=js["kp_fw"],
                force_limit=js["force_limit"])
            buf["previous_motor"] = raw.clone()
            buf["previous_applied"] = motor[:, :, 0].clone()
            self.native.step_motor(motor.contiguous(), torch.zeros(n, 3, device=target.device, dtype=target.dtype))
            f = self._frames()
            buf["joints"] = f["joints"]
            stats = self.native.self_contact_stats()
            buf["self_contacts"] = torch.maximum(buf["self_contacts"], stats[:, 0])
            buf["self_penetration"] = torch.maximum(buf["self_penetration"], stats[:, 1])
            if cfg.mean_velocity_tau:
                alpha = -math.expm1(-cfg.dt / cfg.mean_velocity_tau)
                buf["mean_velocity_world"] = buf["mean_velocity_world"].lerp(f["origin_world_velocity"], alpha)
            buf["air_time"] = torch.where(f["contact"], 0.0, buf["air_time"] + cfg.dt)
            buf["contact_time"] = torch.where(f["contact"], buf["contact_time"] + cfg.dt, 0.0)
        buf["episode_length_buf"] = buf["episode_length_buf"] + 1
        self.common_step_counter += 1
        f["air_time"] = buf["air_time"]
        reward = torch.zeros(n, device=target.device)
        terms = {}
        if self.reward_enabled:
            features = dict(
                command=buf["command"], lin_vel=f["lin_vel"], ang_vel=f["ang_vel"], gravity=f["gravity"],
                world_ang_vel=f["bodies"][:, 1, 10:13], angular_momentum=angular_momentum(f["bodies"], cfg),
                joint_pos=f["joints"][:, :, 0], action=buf["action"], previous_action=buf["old_action"],
                contact=f["contact"], contact_time=buf["contact_time"], air_time=buf["air_time"],
                foot_height=f["site_pos"][:, :, 2], foot_vel=f["site_vel"], episode_steps=buf["episode_length_buf"],
                head_command=torch.zeros_like(self.reward.head_ema), self_collisions=buf["self_contacts"])
            terms = self.reward.terms(features, cfg.step_dt)
            weights = walking_weights(self.source_iteration + self.common_step_counter // 24)
            weights.update(cfg.reward_weight_overrides)
            hs = self.head_stability
            if hs:
                terms["head_position_l2"] = (f["joints"][:, cfg.head_ids, 0] - cfg.home[:, cfg.head_ids]).square().sum(-1)
                terms["head_velocity_l2"] = f["joints"][:, cfg.head_ids, 1].square().sum(-1)
                weights["head_position_l2"] = -hs["position_weight"]
                weights["head_velocity_l2"] = -hs["velocity_weight"]
            if cfg.mean_velocity_tau:
                local_mean = inverse_rotate(f["root_quat"], buf["mean_velocity_world"])
                terms["track_mean_velocity"] = torch.exp(-((local_mean[:, :2] - buf["command"][:, :2]).square().sum(-1))
                                                         / cfg.training["mean_velocity_variance"])
                weights["track_mean_velocity"] = cfg.training["mean_velocity_weight"]
            if cfg.heading_reward_weight:
                terms["track_heading"] = torch.exp(-heading_error(buf["target_yaw"], f["root_quat"]).square()
                                                   / cfg.training["heading_reward_variance"])
                weights["track_heading"] = cfg.heading_reward_weight
            reward = sum(weights[name] * value for name, value in terms.items()) * cfg.step_dt
        timeout = buf["episode_length_buf"] >= cfg.max_episode_length
        failed = failure(f["gravity"], f["diag"], buf["self_penetration"], f["joints"])
        done = failed | timeout
        if cfg.heading_hold:
            buf["command"][:, 2] = (0.5 * heading_error(buf["target_yaw"], f["root_quat"])).clamp(-1.0, 1.0)
        heading = heading_error(buf["target_yaw"], f["root_quat"]) if cfg.heading_reward_weight else None
        obs = observations(f, f["joints"], cfg.home, buf["observed_velocity"], buf["action"], buf["command"],
                           buf["mean_velocity_world"] if cfg.mean_velocity_tau else None, heading)
        return dict(obs=obs, reward=reward.float(), done=done, timeout=timeout, failed=failed, terms=terms,
                    frames=f)


def config_from_bundle(config_json: dict, model_text: str, num_envs: int, *, dt: float, step_dt: float,
                       max_episode_length: int, training: dict | None = None, heading_hold=False,
                       dtype=torch.float32, device="cpu") -> BamConfig:
    """BamConfig of a BAM bundle as the reference BamEnv builds it
    (bam_env.py:33-133)."""
    training = training or {}
    t = lambda x: torch.as_tensor(x, dtype=dtype, device=device)
    mass, inertia = body_table(model_text, dtype)
    return BamConfig(
        home=t(config_json["default_qpos"][7:]).expand(num_envs, -1).clone(),
        root_offset=t(config_json["root_com_offset"]).expand(num_envs, -1).contiguous(),
        root_rotation_inv=t(config_json["root_principal_quat"]) * t([1, -1, -1, -1]),
        foot_ids=[f["body"] for f in config_json["feet"]],
        foot_sites=t([f["site"] for f in config_json["feet"]]),
        mass=mass.to(device), inertia=inertia.to(device),
        soft_limits=soft_limits_from_model(model_text, num_envs, dtype).to(device),
        joint_names=list(config_json["joint_names"]), dt=dt, step_dt=step_dt,
        max_episode_length=max_episode_length,
        mean_velocity_tau=training.get("mean_velocity_tau", 0.0),
        heading_reward_weight=training.get("heading_reward_weight", 0.0),
        heading_hold=training.get("heading_hold", heading_hold),
        linear_variance=training.get("horizontal_velocity_variance", 0.1),
        vertical_variance=training.get("vertical_velocity_variance", 0.1),
        training=training or None,
        reward_weight_overrides=training.get("reward_weight_overrides", {}))
