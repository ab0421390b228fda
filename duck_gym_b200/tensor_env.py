"""Tensor VecEnv over the B200 batch: drop-in for the reference's
``python/duck_gym/tensor_env.py`` ``TensorEnv`` (rsl-rl VecEnv contract:
``reset(mask)``, ``step(actions) -> (obs, reward, done, info)``,
``get_observations()``), same constructor arguments and buffers.

Each control step runs as four kernels instead of the reference's ~60 torch
ops plus physics: ``duck_env_targets`` (clamped action -> PD target), the
physics step, ``duck_env_post_step`` (frames, termination, reward, time-outs,
bookkeeping and terminal observation, read straight from the physics state),
and ``duck_env_observe`` after the auto-reset.  Reset draws its noise with the
reference's generator calls, so it reproduces the reference env's draws on the
same device.

Supported: tasks "standing" and "locomotion", the velocity filter, fixed or
random command directions, the gait reference, foot-clearance and
load-transfer shaping (from the ``gait.npz`` next to the model, as in the
reference), fp32 and fp64.  There is no CPU backend: the CPU path of the
reference is its own solver.
"""

from __future__ import annotations

import ctypes
import json
import math
from pathlib import Path

import torch

from .cuda_batch import CudaBatch, _raise, library


class EnvParams(ctypes.Structure):
    _fields_ = [("task", ctypes.c_int), ("filter", ctypes.c_int), ("max_episode_length", ctypes.c_int),
                ("root_height", ctypes.c_double), ("tilt", ctypes.c_double), ("control_dt", ctypes.c_double),
                ("velocity_alpha", ctypes.c_double), ("tracking_weight", ctypes.c_double),
                ("heading_weight", ctypes.c_double), ("tracking_sigma", ctypes.c_double),
                ("gait_period", ctypes.c_double), ("iquat", ctypes.c_double * 4),
                ("gait", ctypes.c_int), ("foot_clearance", ctypes.c_int), ("load_transfer", ctypes.c_int),
                ("gait_samples", ctypes.c_int), ("foot_points", ctypes.c_int), ("foot_body", ctypes.c_int * 2),
                ("gait_lift", ctypes.c_double), ("mass", ctypes.c_double),
                ("gait_table", ctypes.c_void_p), ("foot_xyz", ctypes.c_void_p)]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


class TensorEnv:
    def __init__(self, model_dir, num_envs=128, iterations=200, dt=0.001, substeps=20, seed=42,
                 action_scale=0.3, episode_seconds=30, task="standing", randomize=True, auto_reset=True,
                 fp64=False, command_speed=0.05, backend="cuda", cpu_threads=1, gait=False,
                 foot_clearance=False, tracking_sigma=None, load_transfer=False, velocity_filter_seconds=0.0,
                 tracking_weight=4.0, heading_weight=0.4, command_direction="all", device=0):
        # Argument validation follows tensor_env.py:85-176.
        if substeps < 1 or episode_seconds <= 0 or action_scale <= 0:
            raise ValueError("Invalid control configuration")
        if backend not in ("cpu", "cuda"):
            raise ValueError(backend)
        if backend != "cuda":
            raise ValueError("duck_gym_b200 runs on CUDA only; the CPU path is the reference's own solver")
        self.device = torch.device("cuda", device)
        self.num_envs = num_envs
        self.num_actions = 14
        self.dtype = torch.float64 if fp64 else torch.float32
        self.model_dir = Path(model_dir)
        self.meta = json.loads((self.model_dir / "metadata.json").read_text())
        self._gait_record = None
        if gait or foot_clearance or load_transfer:
            import numpy as np

            self._gait_record = np.load(self.model_dir / "gait.npz")
        self.native = CudaBatch(str(self.model_dir / "microduck.duck"), num_envs, dt, iterations, device, fp64)
        if self.native.joint_names != self.meta["joint_names"]:
            raise ValueError("Joint order mismatch")
        self.num_actions = self.native.num_joints
        if task not in ("standing", "locomotion"):
            raise ValueError(task)
        self.task = task
        if any(not math.isfinite(x) or x < 0 for x in (tracking_weight, heading_weight)):
            raise ValueError("Reward weights must be finite and nonnegative")
        self.tracking_weight = tracking_weight
        self.heading_weight = heading_weight
        self.randomize = randomize
        self.auto_reset = auto_reset
        self.velocity_filter_seconds = velocity_filter_seconds
        if not math.isfinite(velocity_filter_seconds) or velocity_filter_seconds < 0:
            raise ValueError("velocity filter must be nonnegative")
        if velocity_filter_seconds > 0 and task != "locomotion":
            raise ValueError("Velocity filter is for locomotion")
        self.control_dt = dt * substeps
        self.velocity_alpha = (1 - math.exp(-self.control_dt / velocity_filter_seconds)
                               if velocity_filter_seconds > 0 else 1.0)
        self.substeps = substeps
        self.action_scale = action_scale
        self.max_episode_length = round(episode_seconds / self.control_dt)
        self.gait, self.foot_clearance, self.load_transfer = gait, foot_clearance, load_transfer
        self.gait_period = 0.8
        self.tracking_sigma = tracking_sigma if tracking_sigma is not None else (0.02 if gait else 0.04)
        if self.tracking_sigma <= 0:
            raise ValueError("tracking sigma must be positive")
        self.command_speed = command_speed
        if gait or foot_clearance or load_transfer:
            # tensor_env.py:152-171: the gait record prepared next to the model.
            record = self._gait_record
            self.gait_table = torch.tensor(record["targets"], device=self.device, dtype=self.dtype).contiguous()
            self.gait_period = float(record["period"])
            self.gait_lift = float(record["lift"]) if "lift" in record.files else 0.008
            self.foot_points = torch.tensor(record["foot_collision_points"], device=self.device,
                                            dtype=self.dtype).contiguous()
            self.foot_bodies = torch.tensor(record["foot_bodies"], device=self.device, dtype=torch.long)
            if abs(float(record["speed"]) - command_speed) > 1e-8:
                raise ValueError("Gait command speed mismatch")
            self.gait_directions = torch.tensor([[1.0, 0], [-1, 0], [0, 1], [0, -1]], device=self.device,
                                                dtype=self.dtype)
        self.direction_names = ("forward", "backward", "left", "right")
        if command_direction not in ("all", *self.direction_names):
            raise ValueError("Invalid command direction")
        self.command_direction = command_direction
        dev, dt_ = self.device, self.dtype
        self.episode_length_buf = torch.zeros(num_envs, device=dev, dtype=torch.long)
        self.generator = torch.Generator(device=dev).manual_seed(seed)
        self.home = torch.tensor(self.meta["home"], device=dev, dtype=dt_)
        self.lower = torch.tensor(self.meta["lower"], device=dev, dtype=dt_)
        self.upper = torch.tensor(self.meta["upper"], device=dev, dtype=dt_)
        self.iquat = torch.tensor(self.meta["root_iquat"], device=dev, dtype=dt_) * torch.tensor(
            [1, -1, -1, -1], device=dev)
        self.actions = torch.zeros(num_envs, self.num_actions, device=dev, dtype=dt_)
        self.forces = torch.zeros(num_envs, 3, device=dev, dtype=dt_)
        self.commands = torch.zeros(num_envs, 2, device=dev, dtype=dt_)
        self.filtered_velocity = torch.zeros(num_envs, 2, device=dev, dtype=dt_)
        self.returns = torch.zeros(num_envs, device=dev)
        self._directions = torch.tensor([[1.0, 0], [-1, 0], [0, 1], [0, -1]], device=dev, dtype=dt_)
        # Work buffers of the fused step.
        self._a = torch.zeros_like(self.actions)
        self._target = torch.zeros_like(self.actions)
        self._params = EnvParams(
            task=1 if task == "locomotion" else 0, filter=int(velocity_filter_seconds > 0),
            max_episode_length=self.max_episode_length, root_height=self.meta["root_height"],
            tilt=float(-torch.cos(torch.tensor(0.5, device=dev))), control_dt=self.control_dt,
            velocity_alpha=self.velocity_alpha, tracking_weight=tracking_weight, heading_weight=heading_weight,
            tracking_sigma=self.tracking_sigma, gait_period=self.gait_period,
            iquat=(ctypes.c_double * 4)(*[float(v) for v in self.iquat.cpu()]))
        if gait or foot_clearance or load_transfer:
            p = self._params
            p.gait, p.foot_clearance, p.load_transfer = int(gait), int(foot_clearance), int(load_transfer)
            p.gait_samples, p.foot_points = self.gait_table.shape[1], self.foot_points.shape[1]
            p.foot_body = (ctypes.c_int * 2)(*[int(v) for v in self.foot_bodies.tolist()])
            p.gait_lift, p.mass = self.gait_lift, float(self.meta["mass"])
            p.gait_table, p.foot_xyz = self.gait_table.data_ptr(), self.foot_points.data_ptr()
        self._lib = library()
        self.num_obs = self._lib.duck_env_obs_dim(self.native._h, ctypes.byref(self._params))
        self.reset(torch.ones(num_envs, device=dev, dtype=torch.bool))

    # ---------------------------------------------------------------- helpers
    @property
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _observe(self):
        obs = torch.empty(self.num_envs, self.num_obs, device=self.device)
        _raise(self._lib.duck_env_observe(self.native._h, ctypes.byref(self._params), _ptr(self.home),
                                          _ptr(self.actions), _ptr(self.episode_length_buf), _ptr(self.commands),
                                          _ptr(self.filtered_velocity), _ptr(obs), self._stream))
        return obs

    # ---------------------------------------------------------------- API
    def reset(self, mask):
        """tensor_env.py:178-219 (same generator draws)."""
        mask = mask.to(self.device, torch.bool).contiguous()
        q = self.home.expand(self.num_envs, -1).clone()
        roots = torch.zeros(self.num_envs, 6, device=self.device, dtype=self.dtype)
        if self.randomize:
            q += (torch.rand(q.shape, generator=self.generator, device=self.device, dtype=self.dtype) - 0.5) * 0.02
            roots[:, 3:5] = (torch.rand((self.num_envs, 2), generator=self.generator, device=self.device,
                                        dtype=self.dtype) - 0.5) * 0.02
            roots[:, 2] = 0.001
        self.native.reset(mask, q.contiguous(), roots)
        new_commands = None
        if self.task == "locomotion":
            if self.command_direction == "all":
                selected = torch.randint(4, (self.num_envs,), generator=self.generator, device=self.device)
            else:
                selected = torch.full((self.num_envs,), self.direction_names.index(self.command_direction),
                                      device=self.device, dtype=torch.long)
            new_commands = (self._directions[selected] * self.command_speed).contiguous()
        _raise(self._lib.duck_env_reset_buffers(self.native._h, _ptr(mask), _ptr(self.actions), _ptr(self.forces),
                                                _ptr(self.episode_length_buf), _ptr(self.returns),
                                                _ptr(self.filtered_velocity), _ptr(self.commands),
                                                _ptr(new_commands), self._stream))

    def state(self):
        """tensor_env.py:221-236 (torch frame math over a state snapshot)."""
        from .frames import multiply, inverse_rotate

        b, j, d = [v.to(self.dtype) for v in self.native.state()]
        q = multiply(b[:, 1, 3:7], self.iquat.expand(self.num_envs, -1))
        down = torch.tensor([0.0, 0, -1], device=self.device, dtype=self.dtype).expand(self.num_envs, -1)
        gravity = inverse_rotate(q, down)
        v = inverse_rotate(q, b[:, 1, 7:10])
        w = inverse_rotate(q, b[:, 1, 10:13])
        yaw = torch.stack((1 - 2 * (q[:, 2] ** 2 + q[:, 3] ** 2), 2 * (q[:, 0] * q[:, 3] + q[:, 1] * q[:, 2])), dim=-1)
        return b, j, d, gravity, v, w, yaw

    def observations(self, state):
        """tensor_env.py:238-258, from a ``state()`` tuple (torch ops; the step
        itself uses the fused kernel)."""
        b, j, d, g, v, w, yaw = state
        pieces = [g, v, w, b[:, 1, 2:3] - self.meta["root_height"], j[:, :, 0] - self.home, 0.1 * j[:, :, 1],
                  self.actions]
        if self.task == "locomotion":
            phase = self.episode_length_buf.to(self.dtype) * self.control_dt * (2 * torch.pi / self.gait_period)
            pieces.extend([self.commands, yaw, torch.stack((phase.sin(), phase.cos()), dim=-1)])
        if self.velocity_filter_seconds > 0:
            pieces.append(self.filtered_velocity)
        return torch.cat(pieces, dim=-1).float()

    def get_observations(self):
        return self._observe(), {"observations": {}}

    def reference(self):
        """tensor_env.py:263-277 (torch ops; the step uses the fused kernel)."""
        if not self.gait:
            return self.home.expand(self.num_envs, -1)
        phase = self.episode_length_buf.to(self.dtype) * self.control_dt / self.gait_period
        count = self.gait_table.shape[1]
        index = (phase % 1) * count
        lo = index.long()
        fraction = (index - lo)[:, None]
        direction = (self.commands @ self.gait_directions.T).argmax(-1)
        ref = (self.gait_table[direction, lo] * (1 - fraction)
               + self.gait_table[direction, (lo + 1) % count] * fraction)
        blend = (self.episode_length_buf.to(self.dtype) * self.control_dt).clamp(0, 1)[:, None]
        return self.home + (ref - self.home) * blend

    def step(self, actions):
        """tensor_env.py:279-391."""
        lib, h, stream = self._lib, self.native._h, self._stream
        n = self.num_envs
        acts = actions.to(self.device, self.dtype).contiguous()
        if self.gait:
            _raise(lib.duck_env_reference_targets(
                h, ctypes.byref(self._params), _ptr(acts), float(self.action_scale), _ptr(self.home),
                _ptr(self.lower), _ptr(self.upper), _ptr(self.episode_length_buf), _ptr(self.commands),
                _ptr(self._a), _ptr(self._target), stream))
        else:
            _raise(lib.duck_env_targets(h, _ptr(acts), float(self.action_scale), _ptr(self.home), _ptr(self.lower),
                                        _ptr(self.upper), _ptr(self._a), _ptr(self._target), stream))
        self.native.step(self._target, self.forces, self.substeps, self.meta["kp"], self.meta["torque_limit"])
        obs = torch.empty(n, self.num_obs, device=self.device)
        reward = torch.empty(n, device=self.device)
        failed = torch.empty(n, device=self.device, dtype=torch.bool)
        timeout = torch.empty_like(failed)
        done = torch.empty_like(failed)
        diag = torch.empty(n, 6, device=self.device, dtype=self.dtype)
        tracking = torch.empty(n, 4, device=self.device) if self.task == "locomotion" else None
        _raise(lib.duck_env_post_step(h, ctypes.byref(self._params), _ptr(self.home), _ptr(self._a),
                                      _ptr(self.actions), _ptr(self.episode_length_buf), _ptr(self.returns),
                                      _ptr(self.commands), _ptr(self.filtered_velocity), _ptr(obs), _ptr(reward),
                                      _ptr(failed), _ptr(timeout), _ptr(done), _ptr(diag), _ptr(tracking), stream))
        info = {
            "observations": {},
            "time_outs": timeout,
            "failed": failed,
            "diagnostics": diag,
            "applied_targets": self._target.clone(),
            "terminal_observation": obs,
            "terminal_mask": done,
            "log": {
                "physics/failed_fraction": failed.float().mean(),
                "physics/max_joint_error_m": diag[:, 0].max(),
                "physics/max_penetration_m": diag[:, 1].max(),
            },
        }
        if tracking is not None:
            means = tracking.mean(0)
            info["log"].update({
                "tracking/instant_error_mps": means[0],
                "tracking/command_direction_mps": means[1] / max(self.command_speed, 1e-8),
                "tracking/reward_velocity_error_mps": means[2],
                "tracking/absolute_yaw_rad": means[3],
            })
        if self.auto_reset:
            self.reset(done)
            obs = self.get_observations()[0]
        return obs, reward, done, info
