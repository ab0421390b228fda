"""GPU: the fused BAM environment (``duck_bam_*`` through the C ABI, driven by
``duck_gym_b200.BamEnv``) against the BAM restatement
(``oracle/bam_math.BamStepper``), teacher-forced one control step at a time.

The checker runs the restated step on the CPU over a second GPU batch that
holds the same physics state.  For every substep the servo output of the
restatement must match the fused servo's motor channels; the checker then
steps its batch with the fused channels, so both physics states stay
identical and every later quantity is compared on the same state.

Bar: done / time-out / failure masks and episode counters bit exact; motor
channels, observations, rewards and reward terms within float rounding
(tolerances below).  The CUDA-graph replay is bit-identical to eager launches.
"""

import json

import numpy as np
import pytest
import torch

from oracle import bam_math

pytestmark = pytest.mark.gpu

MOTOR_TOL = dict(rtol=1e-4, atol=1e-6)
OBS_TOL = dict(rtol=2e-5, atol=2e-6)
COMMANDS = [[0.05, 0.0, 0.0], [-0.05, 0.0, 0.0], [0.0, 0.05, 0.0], [0.0, -0.05, 0.0], [0.0, 0.0, 0.0]]
# The key sets of the reference's native_bam_head_stability.json and
# native_bam_heading.json training dictionaries.
TRAININGS = {
    "head_stability": dict(commands=COMMANDS, command_resample_seconds=0.2, reset_joint_noise=0.01,
                           reset_tilt_noise=0.01, horizontal_velocity_variance=0.1, vertical_velocity_variance=0.1,
                           mean_velocity_tau=0.5, mean_velocity_variance=0.0025, mean_velocity_weight=4.0,
                           heading_hold=True, reward_weight_overrides={"self_collisions": -5.0,
                                                                       "head_pose_tracking": 4.0},
                           head_stability={"position_weight": 8.0, "velocity_weight": 0.04}),
    "heading": dict(commands=COMMANDS, command_resample_seconds=0.2, reset_joint_noise=0.01, reset_tilt_noise=0.01,
                    horizontal_velocity_variance=0.0025, vertical_velocity_variance=0.1, mean_velocity_tau=0.5,
                    mean_velocity_variance=0.0025, mean_velocity_weight=4.0, heading_hold=True,
                    heading_reward_weight=2.0, heading_reward_variance=0.04, neutral_head=True),
}


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


@pytest.fixture(scope="module")
def bundle(tmp_path_factory):
    from duck_gym_b200 import biped

    return biped.write_bam(tmp_path_factory.mktemp("bam"), seed=0)


class ForcedEngine:
    """The checker's physics: a second GPU batch, read back to the CPU.  Its
    motor input is checked against, then replaced by, the fused path's."""

    def __init__(self, batch, motors):
        self.b, self.motors, self.k = batch, motors, 0
        self.zeros = torch.zeros(batch.num_envs, 3, device=batch.device, dtype=batch.dtype)

    def generalized_loads(self, offset):
        return self.b.generalized_loads(offset.to(self.b.device).contiguous()).cpu()

    def step_motor(self, motor, forces):
        fused = self.motors[self.k]
        self.k += 1
        torch.testing.assert_close(motor, fused.cpu(), **MOTOR_TOL)
        self.b.step_motor(fused, self.zeros)

    def state(self):
        return tuple(t.cpu() for t in self.b.state())

    def contact_forces(self, ground_only=False):
        return self.b.contact_forces(ground_only).cpu()

    def self_contact_stats(self):
        return self.b.self_contact_stats().cpu()


def checker_for(env, training):
    cfg = bam_math.config_from_bundle(env.cfg, (env_model_text(env)), env.num_envs, dt=env.dt, step_dt=env.step_dt,
                                      max_episode_length=env.max_episode_length, training=training, dtype=env.dtype)
    return bam_math.BamStepper(None, cfg, env.cfg, env.lag, env.decimation, reward_enabled=env.reward_enabled,
                               source_iteration=env.source_iteration, neutral_head=env.neutral_head,
                               head_stability=training.get("head_stability"))


def env_model_text(env):
    return (env._model_dir / "model.duck").read_text()


def env_buffers(env):
    names = ("action", "old_action", "previous_motor", "previous_applied", "observed_velocity", "command",
             "mean_velocity_world", "target_yaw", "air_time", "contact_time", "episode_length_buf", "target_history",
             "history_initialized", "self_contacts", "self_penetration", "joints")
    out = {n: getattr(env, n).detach().cpu().clone() for n in names}
    out["head_ema"] = env.reward_model.head_ema.cpu().clone()
    out["peak_height"] = env.reward_model.peak_height.cpu().clone()
    return out


@pytest.mark.parametrize("case", list(TRAININGS))
def test_bam_step_matches_restatement(bundle, case):
    from duck_gym_b200 import CudaBatch
    from duck_gym_b200.bam_env import BamEnv, TERM_NAMES

    training = TRAININGS[case]
    env = BamEnv(bundle, num_envs=32, iterations=10, auto_reset=True, seed=3, reward_enabled=True,
                 training=training, seconds=0.3, source_iteration=749)
    twin = CudaBatch(str(bundle / "model.duck"), env.num_envs, env.dt, 10, 0, False)
    st = checker_for(env, training)
    gen = torch.Generator().manual_seed(23)
    failures = timeouts = 0
    for step in range(30):
        actions = (torch.rand(env.num_envs, 14, generator=gen) * 2.4 - 1.2).cuda()
        twin.import_records(env.native.export_records())
        st.load(env_buffers(env), env.history_cursor, env.common_step_counter)
        motors = []
        obs, reward, done, info = env.step(actions, substep_callback=lambda e: motors.append(e._motor.clone()))
        st.native = ForcedEngine(twin, motors)
        out = st.step(actions.cpu())
        assert st.native.k == env.decimation
        for key, got in (("done", done.bool()), ("timeout", info["time_outs"]), ("failed", env.failure_mask())):
            assert torch.equal(got.cpu(), out[key]), f"{case} step {step} {key}"
        torch.testing.assert_close(reward.cpu(), out["reward"], **OBS_TOL)
        terminal = info["terminal_observation"]
        torch.testing.assert_close(terminal["actor"].cpu(), out["obs"]["actor"], **OBS_TOL)
        torch.testing.assert_close(terminal["critic"].cpu(), out["obs"]["critic"], **OBS_TOL)
        for name, value in out["terms"].items():
            torch.testing.assert_close(info["log"][f"Reward/{name}"].cpu().double(), value.double().mean(),
                                       rtol=2e-5, atol=1e-6, msg=f"{case} step {step} {name}")
        assert set(f"Reward/{n}" for n in out["terms"]) <= set(info["log"])
        failures += int(out["failed"].sum())
        timeouts += int(out["timeout"].sum())
    assert failures > 0 and timeouts > 0
    assert TERM_NAMES[0] == "track_linear_velocity"


def test_bam_graph_replay_is_bit_identical_to_eager(bundle):
    from duck_gym_b200.bam_env import BamEnv

    training = TRAININGS["head_stability"]
    envs = [BamEnv(bundle, num_envs=16, iterations=10, auto_reset=True, seed=9, reward_enabled=True,
                   training=training, seconds=0.2, use_graph=g) for g in (True, False)]
    gen = torch.Generator().manual_seed(5)
    for _ in range(12):
        actions = (torch.rand(16, 14, generator=gen) * 1.6 - 0.8).cuda()
        outs = [e.step(actions) for e in envs]
        (o1, r1, d1, i1), (o2, r2, d2, i2) = outs
        assert torch.equal(r1, r2) and torch.equal(d1, d2)
        assert torch.equal(o1["actor"], o2["actor"]) and torch.equal(o1["critic"], o2["critic"])
        assert torch.equal(i1["terminal_observation"]["critic"], i2["terminal_observation"]["critic"])
    assert envs[0]._graph is not None and envs[1]._graph is None
    assert torch.equal(envs[0].native.export_records(), envs[1].native.export_records())


def test_bam_reset_draws_match_reference_generator(bundle):
    """Reset noise and commands follow the reference's generator calls
    (bam_env.py:225-251): joint noise, tilt noise, then command indices."""
    from duck_gym_b200.bam_env import BamEnv

    training = TRAININGS["heading"]
    env = BamEnv(bundle, num_envs=24, iterations=10, seed=41, training=training)
    gen = torch.Generator(device="cuda").manual_seed(41)
    home = env.home
    q = home + (torch.rand(home.shape, generator=gen, device="cuda") * 2 - 1) * 0.01
    torch.rand((24, 2), generator=gen, device="cuda")
    idx = torch.randint(len(COMMANDS), (24,), generator=gen, device="cuda")
    commands = torch.tensor(COMMANDS, device="cuda")[idx]
    torch.testing.assert_close(env.joints[:, :, 0], q, rtol=0, atol=2e-5)
    torch.testing.assert_close(env.command[:, :2], commands[:, :2])
    # Heading hold replaced the yaw command by the (zero) heading error.
    assert torch.all(env.command[:, 2].abs() < 1e-6)
    assert (env.episode_length_buf == 0).all() and not env.pending.any()


def test_bam_pending_reset_guard(bundle):
    from duck_gym_b200.bam_env import BamEnv

    env = BamEnv(bundle, num_envs=4, iterations=10, auto_reset=False, seconds=0.04)
    zeros = torch.zeros(4, 14, device="cuda")
    env.step(zeros)
    _, _, done, info = env.step(zeros)
    assert info["time_outs"].all() and done.all()
    with pytest.raises(RuntimeError):
        env.step(zeros)
    env.reset(done.bool())
    env.step(zeros)
