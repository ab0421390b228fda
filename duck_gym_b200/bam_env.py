"""BAM environment over the B200 batch: drop-in for the reference's
``python/duck_gym/bam_env.py`` ``BamEnv`` (the XL330/m6 servo of
``actuator.py`` driving the native engine through its motor channels, the
walking reward of ``walking_reward.py``), same constructor arguments,
buffers and ``reset`` / ``step`` / ``get_observations`` contract.

A control step is one C call, ``duck_bam_step``: a prologue kernel, then per
physics substep the servo kernel (delay ring, RNEA generalized loads, servo
equations), one physics substep and a bookkeeping kernel (foot contacts,
timers, self-contact maxima, mean-velocity filter), then one kernel for
frames, reward terms, failure, time-outs and both observations.  It only
launches kernels, so after the first (eager) step it is captured into a CUDA
graph and replayed.  Resets draw their noise and commands with the
reference's generator calls in the reference's order and run eagerly.

``substep_callback`` is honoured: with a callback the step runs substep by
substep (no graph) and refreshes the frames before each call.  There is no
CPU backend: the reference's CPU path is its own solver.
"""

from __future__ import annotations

import ctypes
import json
import math
from pathlib import Path

import torch

from .cuda_batch import CudaBatch, _raise, library

TERM_NAMES = ("track_linear_velocity", "track_angular_velocity", "upright", "pose", "body_ang_vel",
              "angular_momentum", "dof_pos_limits", "action_rate_l2", "air_time", "foot_clearance",
              "foot_swing_height", "foot_slip", "self_collisions", "head_pose_tracking", "head_pose_bias",
              "head_position_l2", "head_velocity_l2", "track_mean_velocity", "track_heading")
# walking_reward.py:31-37: per-joint pose tolerances when standing / walking.
POSE_STD = dict(hip_yaw=(0.1, 0.3), hip_roll=(0.05, 0.05), hip_pitch=(0.15, 0.4), knee=(0.15, 0.4),
                ankle=(0.1, 0.25))
SERVO_KEYS = ("kt", "R", "friction_base", "friction_stribeck", "load_friction_external", "load_friction_motor",
              "load_friction_external_stribeck", "load_friction_motor_stribeck", "load_friction_external_quad",
              "load_friction_motor_quad", "dtheta_stribeck", "alpha", "friction_viscous")
FEATURES = dict(root_quat=(0, 4), gravity=(4, 7), ang_vel=(7, 10), lin_vel=(10, 13), origin_world_velocity=(13, 16))

_D, _I, _U = ctypes.c_double, ctypes.c_int, ctypes.c_uint32


class BamParams(ctypes.Structure):
    _fields_ = ([(n, _I) for n in ("lag", "decimation", "max_episode_length", "source_iteration", "neutral_head",
                                   "heading_hold", "reward_enabled", "head_stability", "mean_velocity",
                                   "heading_reward")]
                + [("foot_body", _I * 2), ("head_mask", _U), ("override_mask", _U)]
                + [(n, _D) for n in ("dt", "step_dt", "kp_fw", "vin", "vin_drop_gain", "vin_min", "force_limit")]
                + [(n, _D) for n in SERVO_KEYS]
                + [("root_iquat", _D * 4), ("foot_site", (_D * 3) * 2)]
                + [(n, _D) for n in ("linear_variance", "vertical_variance", "mean_velocity_alpha",
                                     "mean_velocity_variance", "mean_velocity_weight", "heading_reward_weight",
                                     "heading_reward_variance", "head_position_weight", "head_velocity_weight",
                                     "tilt_limit")]
                + [("overrides", _D * 15), ("stand_std", _D * 32), ("walk_std", _D * 32),
                   ("soft_limits", (_D * 2) * 32)])


_P = ctypes.c_void_p
BUFFER_NAMES = ("home", "root_offset", "zero_forces", "action", "old_action", "previous_motor", "previous_applied",
                "observed_velocity", "command", "mean_velocity_world", "target_yaw", "self_contacts",
                "self_penetration", "air_time", "contact_time", "peak_height", "contact_force", "joints", "head_ema",
                "target_history", "motor", "features", "terms", "contact", "history_initialized", "done", "timeout",
                "failed", "episode_length", "counters", "obs_actor", "obs_critic", "reward", "servo_supply")


class BamBufferTable(ctypes.Structure):
    _fields_ = [(n, _P) for n in BUFFER_NAMES]


class _RewardState:
    """The reward model's state as the reference exposes it
    (``env.reward_model.head_ema`` / ``peak_height`` / ``reset`` /
    ``weights``)."""

    def __init__(self, env):
        self._env = env

    @property
    def head_ema(self):
        return self._env._head_ema

    @property
    def peak_height(self):
        return self._env._peak_height

    def reset(self, mask):
        self._env._head_ema[mask] = 0
        self._env._peak_height[mask] = 0

    @staticmethod
    def weights(iteration):
        """walking_reward.py:98-122."""
        action = -0.1
        for start, w in ((500, -0.2), (750, -0.4), (1000, -0.6), (1250, -0.8), (1500, -1.0)):
            if iteration >= start:
                action = w
        head = 0.0
        for start, w in ((600, 1.0), (1000, 2.0), (1500, 3.0)):
            if iteration >= start:
                head = w
        return dict(zip(TERM_NAMES[:15], (2.0, 2.0, 2.0, 1.0, -0.05, -0.02, -1.0, action, 3.0, -2.0, -0.25, -0.1,
                                          -1.0, 2.0, head)))


class BamEnv:
    def __init__(self, model_dir, num_envs=1, backend="cuda", fp64=False, iterations=200, auto_reset=False,
                 seconds=40.0, seed=42, reward_enabled=False, source_iteration=0, training=None, heading_hold=False,
                 physics_dt=None, device=0, use_graph=True, max_pairs=32):
        # Validation and settings follow bam_env.py:17-133.
        if backend != "cuda":
            raise ValueError("duck_gym_b200 runs on CUDA only; the CPU path is the reference's own solver")
        self.cfg = json.loads((Path(model_dir) / "config.json").read_text())
        self.device = torch.device("cuda", device)
        self.dtype = torch.float64 if fp64 else torch.float32
        self.num_envs = num_envs
        self.num_actions = 14
        original_dt = self.cfg["physics_dt"]
        self.dt = original_dt if physics_dt is None else float(physics_dt)
        if not math.isfinite(self.dt) or self.dt <= 0:
            raise ValueError("Physics timestep must be positive and finite")
        control_dt = original_dt * self.cfg["decimation"]
        self.decimation = round(control_dt / self.dt)
        if self.decimation < 1 or abs(self.decimation * self.dt - control_dt) > 1e-9:
            raise ValueError("Physics timestep must divide the original control interval")
        self.step_dt = self.dt * self.decimation
        self.max_episode_length = round(seconds / self.step_dt)
        self.auto_reset = auto_reset
        self.reward_enabled = reward_enabled
        self.source_iteration = source_iteration
        self.training = training
        self.heading_hold = (training or {}).get("heading_hold", heading_hold)
        self.heading_reward_weight = (training or {}).get("heading_reward_weight", 0.0)
        if self.heading_reward_weight and not self.heading_hold:
            raise ValueError("Heading reward requires the initial-heading command controller")
        self.mean_velocity_tau = (training or {}).get("mean_velocity_tau", 0.0)
        if self.mean_velocity_tau < 0:
            raise ValueError("Mean velocity time constant must be nonnegative")
        self.common_step_counter = 0
        self.generator = torch.Generator(device=self.device).manual_seed(seed)
        t = lambda x: torch.as_tensor(x, dtype=self.dtype, device=self.device)
        E = num_envs
        self.home = t(self.cfg["default_qpos"][7:]).expand(E, -1).clone()
        self.root_offset = t(self.cfg["root_com_offset"]).expand(E, -1).contiguous()
        self.root_rotation_inv = t(self.cfg["root_principal_quat"]) * t([1, -1, -1, -1])
        self.foot_ids = [f["body"] for f in self.cfg["feet"]]
        self.foot_points = [t(f["points"]) for f in self.cfg["feet"]]
        self.foot_sites = t([f["site"] for f in self.cfg["feet"]])
        self.zeros_force = torch.zeros(E, 3, device=self.device, dtype=self.dtype)
        model = str(Path(model_dir) / "model.duck")
        lines = Path(model).read_text().splitlines()
        body_count = int(lines[0].split()[2])
        body_rows = [line.split() for line in lines[2:2 + body_count]]
        self.mass = t([float(row[1]) for row in body_rows])
        self.inertia = t([[float(v) for v in row[2:5]] for row in body_rows])
        joint_rows = [line.split() for line in lines[2 + body_count:2 + body_count + 14]]
        limits = t([[float(row[22]), float(row[23])] for row in joint_rows])
        center = limits.mean(-1, keepdim=True)
        self.soft_limits = (center + 0.9 * (limits - center))[None, :, :].expand(E, -1, -1)
        self._model_dir = Path(model_dir)
        self.native = CudaBatch(model, E, self.dt, iterations, device, fp64, max_pairs=max_pairs)
        J = self.native.num_joints
        if J != 14 or len(self.foot_ids) != 2:
            raise ValueError("The BAM environment needs the 14-joint biped with two feet")
        zeros = lambda *shape, dtype=None: torch.zeros(*shape, device=self.device, dtype=dtype or self.dtype)
        self.action, self.old_action = zeros(E, J), zeros(E, J)
        self.previous_motor, self.previous_applied = zeros(E, J), zeros(E, J)
        self.previous_velocity, self.observed_velocity = zeros(E, J), zeros(E, J)
        self.command, self.mean_velocity_world = zeros(E, 3), zeros(E, 3)
        self.target_yaw = zeros(E)
        self.air_time, self.contact_time = zeros(E, 2), zeros(E, 2)
        self.episode_length_buf = zeros(E, dtype=torch.long)
        self.pending = zeros(E, dtype=torch.bool)
        lag_seconds = round(sum(self.cfg["delay_lag_steps"]) / 2) * original_dt
        self.lag = round(lag_seconds / self.dt)
        if abs(self.lag * self.dt - lag_seconds) > 1e-9:
            raise ValueError("Physics timestep must preserve the original actuator lag")
        self.target_history = self.home[None, :, :].expand(self.lag + 1, -1, -1).clone()
        self.history_initialized = zeros(E, dtype=torch.bool)
        self.head_ids = [i for i, n in enumerate(self.cfg["joint_names"]) if "head" in n or "neck" in n]
        self.neutral_head = (training or {}).get("neutral_head", False)
        self.leg_ids = [i for i in range(14) if i not in self.head_ids]
        self.head_average = zeros(E, 4)
        self.self_contacts, self.self_penetration = zeros(E), zeros(E)
        self.reward_weight_overrides = (training or {}).get("reward_weight_overrides", {})
        unknown = set(self.reward_weight_overrides) - set(_RewardState.weights(0))
        if unknown or any(not math.isfinite(v) for v in self.reward_weight_overrides.values()):
            raise ValueError("Unknown or nonfinite reward weight override")
        linear_variance = (training or {}).get("horizontal_velocity_variance", 0.1)
        vertical_variance = (training or {}).get("vertical_velocity_variance", 0.1)
        if linear_variance <= 0 or vertical_variance <= 0:
            raise ValueError("Velocity variances must be positive")
        self.reward_model = _RewardState(self)
        self._head_ema, self._peak_height = zeros(E, len(self.head_ids)), zeros(E, 2)
        # Buffers only the fused path uses.
        self._joints = zeros(E, J, 2)
        self._contact_force = zeros(E, 2, 3)
        self._contact = zeros(E, 2, dtype=torch.bool)
        self._motor = zeros(E, J, 3)
        self._features = zeros(E, 29)
        self._terms = zeros(E, len(TERM_NAMES))
        self._done, self._timeout, self._failed = (zeros(E, dtype=torch.bool) for _ in range(3))
        self._counters = torch.zeros(2, device=self.device, dtype=torch.int32)
        self._servo_supply = zeros(E)
        self._obs_actor = torch.zeros(E, 19 + 3 * J, device=self.device)
        self._reward = torch.zeros(E, device=self.device)
        self._actions_in = zeros(E, J)
        self._params = self._make_params(training or {}, linear_variance, vertical_variance)
        self._lib = library()
        critic = self._lib.duck_bam_critic_dim(self.native._h, ctypes.byref(self._params))
        self._obs_critic = torch.zeros(E, critic, device=self.device)
        self._table = BamBufferTable(**{n: self._buffer(n).data_ptr() for n in BUFFER_NAMES})
        self._graph = None
        self._use_graph = use_graph
        self._eager_steps = 0
        self.refresh()
        if training is not None:
            self.reset()

    # ------------------------------------------------------------ set-up
    def _buffer(self, name):
        own = {"home": self.home, "root_offset": self.root_offset, "zero_forces": self.zeros_force,
               "target_history": self.target_history, "episode_length": self.episode_length_buf,
               "history_initialized": self.history_initialized, "joints": self._joints,
               "contact_force": self._contact_force, "contact": self._contact, "motor": self._motor,
               "features": self._features, "terms": self._terms, "done": self._done, "timeout": self._timeout,
               "failed": self._failed, "counters": self._counters, "obs_actor": self._obs_actor,
               "obs_critic": getattr(self, "_obs_critic", None), "reward": self._reward,
               "head_ema": self._head_ema, "peak_height": self._peak_height, "servo_supply": self._servo_supply}
        t = own[name] if name in own else getattr(self, name)
        assert t.is_contiguous() and t.device == self.device
        return t

    def _make_params(self, training, linear_variance, vertical_variance):
        cfg = self.cfg
        p = BamParams()
        p.lag, p.decimation, p.max_episode_length = self.lag, self.decimation, self.max_episode_length
        p.source_iteration = self.source_iteration
        p.neutral_head, p.heading_hold, p.reward_enabled = int(self.neutral_head), int(self.heading_hold), int(
            self.reward_enabled)
        hs = training.get("head_stability", {})
        p.head_stability, p.mean_velocity = int(bool(hs)), int(bool(self.mean_velocity_tau))
        p.heading_reward = int(bool(self.heading_reward_weight))
        p.foot_body = (_I * 2)(*self.foot_ids)
        p.head_mask = sum(1 << j for j in self.head_ids)
        names = list(TERM_NAMES[:15])
        p.override_mask = sum(1 << names.index(k) for k in self.reward_weight_overrides)
        for k, v in self.reward_weight_overrides.items():
            p.overrides[names.index(k)] = float(v)
        p.dt, p.step_dt = self.dt, self.step_dt
        for k in ("kp_fw", "vin", "vin_drop_gain", "vin_min", "force_limit"):
            setattr(p, k, float(cfg[k]))
        for k in SERVO_KEYS:
            setattr(p, k, float(cfg["parameters"][k]))
        for i, v in enumerate(self.root_rotation_inv.tolist()):
            p.root_iquat[i] = v
        for f, site in enumerate(self.foot_sites.tolist()):
            for i, v in enumerate(site):
                p.foot_site[f][i] = v
        p.linear_variance, p.vertical_variance = linear_variance, vertical_variance
        p.mean_velocity_alpha = -math.expm1(-self.dt / self.mean_velocity_tau) if self.mean_velocity_tau else 0.0
        p.mean_velocity_variance = training.get("mean_velocity_variance", 1.0)
        p.mean_velocity_weight = training.get("mean_velocity_weight", 0.0)
        p.heading_reward_weight = self.heading_reward_weight
        p.heading_reward_variance = training.get("heading_reward_variance", 1.0)
        p.head_position_weight = hs.get("position_weight", 0.0)
        p.head_velocity_weight = hs.get("velocity_weight", 0.0)
        p.tilt_limit = -math.cos(math.radians(70.0))
        joint_names = self.cfg["joint_names"]
        for j in self.leg_ids:
            key = next(k for k in POSE_STD if k in joint_names[j])
            p.stand_std[j], p.walk_std[j] = POSE_STD[key]
        for j, (lo, hi) in enumerate(self.soft_limits[0].tolist()):
            p.soft_limits[j][0], p.soft_limits[j][1] = lo, hi
        return p

    @property
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _call(self, name, *args):
        _raise(getattr(self._lib, name)(self.native._h, ctypes.byref(self._params), ctypes.byref(self._table),
                                        *args, self._stream))

    # ------------------------------------------------------------ frames (refresh attributes)
    def refresh(self):
        """bam_env.py:136-170: frames of the current physics state."""
        self._call("duck_bam_observe", None, 0)

    def _feature(self, name):
        lo, hi = FEATURES[name]
        return self._features[:, lo:hi]

    root_quat = property(lambda self: self._feature("root_quat"))
    gravity = property(lambda self: self._feature("gravity"))
    ang_vel = property(lambda self: self._feature("ang_vel"))
    lin_vel = property(lambda self: self._feature("lin_vel"))
    origin_world_velocity = property(lambda self: self._feature("origin_world_velocity"))
    site_pos = property(lambda self: self._features[:, 16:22].view(self.num_envs, 2, 3))
    site_vel = property(lambda self: self._features[:, 22:28].view(self.num_envs, 2, 3))
    joints = property(lambda self: self._joints)
    contact_force = property(lambda self: self._contact_force)
    contact = property(lambda self: self._contact)

    @property
    def history_cursor(self):
        return int(self._counters[0])

    @property
    def bodies(self):
        return self.native.state()[0]

    @property
    def diagnostics(self):
        return self.native.state()[2]

    @property
    def sole_height(self):
        """bam_env.py:172-183 (torch over a state snapshot)."""
        from .frames import inverse_rotate

        foot = self.bodies[:, self.foot_ids]
        conj = foot[:, :, 3:7] * torch.tensor([1, -1, -1, -1], device=self.device, dtype=self.dtype)
        heights = []
        for i, points in enumerate(self.foot_points):
            world = inverse_rotate(conj[:, i, None, :].expand(-1, len(points), -1),
                                   points[None, :, :].expand(self.num_envs, -1, -1))
            heights.append((world[:, :, 2] + foot[:, i, 2, None]).min(-1).values)
        return torch.stack(heights, -1)

    def get_observations(self):
        """bam_env.py:185-211."""
        self.refresh()
        return {"actor": self._obs_actor.clone(), "critic": self._obs_critic.clone()}

    def yaw(self):
        q = self.root_quat
        return torch.atan2(2 * (q[:, 0] * q[:, 3] + q[:, 1] * q[:, 2]), 1 - 2 * (q[:, 2].square() + q[:, 3].square()))

    def heading_error(self):
        error = self.target_yaw - self.yaw()
        return torch.atan2(error.sin(), error.cos())

    def update_heading_command(self):
        if self.heading_hold:
            self._call("duck_bam_observe", None, 1)

    def resample_commands(self, mask):
        """bam_env.py:213-218 (one draw for every env, masked assignment).
        Extension: a training dictionary with ``command_ranges`` [[lo, hi]] x 3
        draws (vx, vy, yaw rate) uniformly instead of from a command list."""
        ranges = self.training.get("command_ranges")
        if ranges is not None:
            r = self.home.new_tensor(ranges)
            u = torch.rand((self.num_envs, 3), generator=self.generator, device=self.device, dtype=self.dtype)
            fresh = r[:, 0] + (r[:, 1] - r[:, 0]) * u
        else:
            commands = self.home.new_tensor(self.training["commands"])
            indices = torch.randint(len(commands), (self.num_envs,), generator=self.generator, device=self.device)
            fresh = commands[indices]
        self.command.copy_(torch.where(mask[:, None], fresh, self.command))

    def failure_mask(self):
        """bam_env.py:409-418, as evaluated at the end of the last step."""
        return self._failed.clone()

    def reward_features(self):
        """bam_env.py:419-447 (torch over a state snapshot)."""
        from .frames import inverse_rotate

        b = self.bodies
        q = b[:, :, 3:7]
        sign = self.home.new_tensor([1, -1, -1, -1])
        local_w = inverse_rotate(q, b[:, :, 10:13])
        spin = inverse_rotate(q * sign, self.inertia[None, :, :] * local_w)
        com = (b[:, :, :3] * self.mass[None, :, None]).sum(1) / self.mass.sum()
        orbital = torch.linalg.cross(b[:, :, :3] - com[:, None, :], b[:, :, 7:10] * self.mass[None, :, None])
        return dict(command=self.command, lin_vel=self.lin_vel, ang_vel=self.ang_vel, gravity=self.gravity,
                    world_ang_vel=b[:, 1, 10:13], angular_momentum=(spin + orbital).sum(1),
                    joint_pos=self.joints[:, :, 0], action=self.action, previous_action=self.old_action,
                    contact=self.contact, contact_time=self.contact_time, air_time=self.air_time,
                    foot_height=self.site_pos[:, :, 2], foot_vel=self.site_vel, episode_steps=self.episode_length_buf,
                    head_command=torch.zeros_like(self.head_average), self_collisions=self.self_contacts)

    # ------------------------------------------------------------ reset / step
    def reset(self, mask=None, *, joint_noise=None, tilt_noise=None):
        """bam_env.py:225-275 (same generator draws in the same order)."""
        if mask is None:
            mask = torch.ones_like(self.pending)
        mask = mask.to(self.device, torch.bool).contiguous()
        initial = self.home.clone()
        root = torch.zeros(self.num_envs, 6, device=self.device, dtype=self.dtype)
        training = self.training or {}
        joint_noise = training.get("reset_joint_noise", 0.0) if joint_noise is None else joint_noise
        tilt_noise = training.get("reset_tilt_noise", 0.0) if tilt_noise is None else tilt_noise
        if joint_noise < 0 or tilt_noise < 0:
            raise ValueError("Reset perturbation amplitudes must be nonnegative")
        if joint_noise or tilt_noise:
            initial += (torch.rand(initial.shape, generator=self.generator, device=self.device, dtype=self.dtype)
                        * 2 - 1) * joint_noise
            root[:, 3:5] = (torch.rand((self.num_envs, 2), generator=self.generator, device=self.device,
                                       dtype=self.dtype) * 2 - 1) * tilt_noise
        if self.training is not None:
            self.resample_commands(mask)
        self.native.reset(mask, initial.contiguous(), root)
        _raise(self._lib.duck_bam_reset_buffers(self.native._h, ctypes.byref(self._params), ctypes.byref(self._table),
                                                ctypes.c_void_p(mask.data_ptr()), self._stream))
        self.head_average.masked_fill_(mask[:, None], 0)
        self.previous_velocity.masked_fill_(mask[:, None], 0)
        self.pending.masked_fill_(mask, False)
        self._call("duck_bam_observe", ctypes.c_void_p(mask.data_ptr()), 1)
        return {"actor": self._obs_actor.clone(), "critic": self._obs_critic.clone()}

    def _capture(self):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._call("duck_bam_step", ctypes.c_void_p(self._actions_in.data_ptr()))
        return graph

    def step(self, actions, *, substep_callback=None):
        """bam_env.py:292-407."""
        if not self.auto_reset and bool(self.pending.any()):
            raise RuntimeError("Reset terminated environments before stepping")
        self._actions_in.copy_(actions.to(self.device, self.dtype))
        if substep_callback is not None:
            self._call("duck_bam_begin", ctypes.c_void_p(self._actions_in.data_ptr()))
            for _ in range(self.decimation):
                self._call("duck_bam_substep")
                self.refresh()
                substep_callback(self)
            self._call("duck_bam_finish")
        elif self._graph is not None:
            self._graph.replay()
        else:
            if self._use_graph and self._eager_steps >= 1:
                # Capture would record (not run) the step: run it eagerly now,
                # then capture once so the next steps replay the graph.  The
                # captured work reads and writes only persistent buffers.
                self._call("duck_bam_step", ctypes.c_void_p(self._actions_in.data_ptr()))
                torch.cuda.synchronize(self.device)
                self._graph = self._capture()
            else:
                self._call("duck_bam_step", ctypes.c_void_p(self._actions_in.data_ptr()))
            self._eager_steps += 1
        self.common_step_counter += 1
        done, timeout = self._done.clone(), self._timeout.clone()
        self.pending.copy_(done)
        reward = self._reward.clone()
        terms = {}
        if self.reward_enabled:
            enabled = list(range(15))
            if self._params.head_stability:
                enabled += [15, 16]
            if self._params.mean_velocity:
                enabled.append(17)
            if self._params.heading_reward:
                enabled.append(18)
            means = self._terms[:, enabled].mean(0)
            terms = {TERM_NAMES[t]: means[i] for i, t in enumerate(enabled)}
        observations = {"actor": self._obs_actor.clone(), "critic": self._obs_critic.clone()}
        info = {
            "time_outs": timeout,
            "terminal_observation": observations,
            "reward_implemented": self.reward_enabled,
            "log": {
                **{f"Reward/{name}": value for name, value in terms.items()},
                "Physics/self_contact_pairs": self.self_contacts.mean(),
                "Physics/self_penetration": self.self_penetration.max(),
                "Physics/numerical_failure": (self._features[:, 28] > 0).float().mean(),
            },
        }
        if self.auto_reset:
            self.reset(done)
            if self.training is not None:
                period = round(self.training["command_resample_seconds"] / self.step_dt)
                self.resample_commands((self.episode_length_buf % period == 0) & ~done)
            # update_heading_command() then get_observations(), in one kernel.
            self._call("duck_bam_observe", None, int(self.heading_hold))
            observations = {"actor": self._obs_actor.clone(), "critic": self._obs_critic.clone()}
        return observations, reward, done.long(), info
