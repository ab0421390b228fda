"""GPU: the fused tensor-environment kernels (``duck_env_*`` through the C
ABI, driven by ``duck_gym_b200.TensorEnv``) against the env-math
restatement (``oracle/env_math.py``) and the reference env's own recorded
outputs (``tests/golden/env_*.npz``).

Bar: failure / time-out / done masks, episode lengths and the velocity filter
state bit exact; observations and rewards within float rounding of the CPU
torch evaluation (OBS_TOL, REWARD_TOL below; fp64 within 1e-12).
"""

import ast
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import env_math

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
OBS_TOL = dict(rtol=1e-5, atol=2e-6)
REWARD_TOL = dict(rtol=1e-5, atol=1e-8)
FP64_TOL = dict(rtol=1e-12, atol=1e-13)


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def make_env(biped_dir, **kw):
    from duck_gym_b200.tensor_env import TensorEnv

    args = dict(num_envs=64, iterations=10, dt=0.005, substeps=4, seed=7)
    args.update(kw)
    return TensorEnv(biped_dir, **args)


def env_config(env):
    cfg = env_math.EnvConfig(
        task=env.task, home=env.home.cpu(), root_height=env.meta["root_height"], root_iquat=env.meta["root_iquat"],
        control_dt=env.control_dt, max_episode_length=env.max_episode_length,
        velocity_filter_seconds=env.velocity_filter_seconds, velocity_alpha=env.velocity_alpha,
        tracking_weight=env.tracking_weight, heading_weight=env.heading_weight, tracking_sigma=env.tracking_sigma,
        tilt=env._params.tilt)
    if env._gait_record is not None:
        env_math.apply_gait(cfg, env._gait_record, env.meta, env.gait, env.foot_clearance, env.load_transfer)
    return cfg


@pytest.fixture(scope="module")
def gait_dir(tmp_path_factory):
    from duck_gym_b200 import biped

    d = tmp_path_factory.mktemp("gait")
    biped.write(d, seed=0)
    biped.write_gait(d, seed=0)
    return d


def snapshot(env):
    return {k: getattr(env, k).detach().cpu().clone() for k in
            ("actions", "episode_length_buf", "returns", "commands", "filtered_velocity")}


def check_step(env, cfg, before, actions, obs, reward, done, info, tol):
    b, j, d = [t.cpu() for t in env.native.state()]
    forces = env.native.contact_forces().cpu()
    a = actions.to(env.dtype).clamp(-1, 1)
    ref = env_math.post_step(b, j, d, a, before["actions"], before["episode_length_buf"], before["returns"],
                             before["commands"], before["filtered_velocity"], cfg, contact_forces=forces)
    if cfg.gait:
        want = (env_math.reference_targets(before["episode_length_buf"], before["commands"], cfg)
                + env.action_scale * a).clamp(env.lower.cpu(), env.upper.cpu())
        torch.testing.assert_close(info["applied_targets"].cpu(), want, **tol["obs"])
    for key, got in (("failed", info["failed"]), ("timeout", info["time_outs"]), ("done", done)):
        assert torch.equal(got.cpu(), ref[key]), key
    assert torch.equal(env.episode_length_buf.cpu(), ref["episode_length"])
    assert torch.equal(env.actions.cpu(), ref["actions"])
    assert torch.equal(info["diagnostics"].cpu(), d)
    if env.velocity_filter_seconds > 0:
        torch.testing.assert_close(env.filtered_velocity.cpu(), ref["filtered"], **tol["obs"])
    torch.testing.assert_close(info["terminal_observation"].cpu(), ref["obs"], **tol["obs"])
    torch.testing.assert_close(reward.cpu(), ref["reward"], **tol["reward"])
    torch.testing.assert_close(env.returns.cpu(), ref["returns"], **tol["reward"])
    return ref


@pytest.mark.parametrize("task,filter_s,scale,fp64,gait", [
    ("standing", 0.0, 0.3, False, False),
    ("locomotion", 0.8, 0.6, False, False),
    ("locomotion", 0.0, 0.6, True, False),
    ("locomotion", 0.0, 0.6, False, True),
])
def test_fused_step_matches_env_math(biped_dir, gait_dir, task, filter_s, scale, fp64, gait):
    env = make_env(gait_dir if gait else biped_dir, task=task, velocity_filter_seconds=filter_s, action_scale=scale,
                   episode_seconds=0.3, fp64=fp64, auto_reset=False, gait=gait, foot_clearance=gait,
                   load_transfer=gait)
    cfg = env_config(env)
    tol = ({"obs": FP64_TOL, "reward": dict(rtol=1e-12, atol=1e-13)} if fp64 else
           {"obs": OBS_TOL, "reward": REWARD_TOL})
    gen = torch.Generator().manual_seed(11)
    failures = timeouts = 0
    for _ in range(30):
        actions = (torch.rand(env.num_envs, env.num_actions, generator=gen) * 2.4 - 1.2).cuda()
        before = snapshot(env)
        obs, reward, done, info = env.step(actions)
        ref = check_step(env, cfg, before, actions.cpu(), obs, reward, done, info, tol)
        failures += int(ref["failed"].sum())
        timeouts += int(ref["timeout"].sum())
        # Auto-reset by hand, then the fresh observation against the restatement.
        env.reset(done)
        fresh = env.get_observations()[0].cpu()
        b, j, d = [t.cpu() for t in env.native.state()]
        g, v, w, yaw = env_math.features(b, cfg)
        want = env_math.observations(b, j, g, v, w, yaw, env.actions.cpu(), env.episode_length_buf.cpu(),
                                     env.commands.cpu(), env.filtered_velocity.cpu(), cfg)
        torch.testing.assert_close(fresh, want, **tol["obs"])
    assert failures > 0 and timeouts > 0


def records_from_golden(bodies, diag, record_length):
    """Portable records holding only what the env math reads: the header
    diagnostics and the body states (no contacts)."""
    E, B, _ = bodies.shape
    rec = np.zeros((E, record_length), dtype=bodies.dtype)
    rec[:, 0] = diag[:, 5]
    rec[:, 2], rec[:, 3], rec[:, 5], rec[:, 6] = diag[:, 0], diag[:, 1], diag[:, 3], diag[:, 4]
    body = rec[:, 8:8 + 16 * B].reshape(E, B, 16)
    body[:, :, :13] = bodies
    rec[:, 8:8 + 16 * B] = body.reshape(E, -1)
    return rec


def test_gait_targets_on_reference_states(gait_dir):
    """The reference env's recorded applied targets (gait table, blend,
    clamp) from the recorded buffers, through duck_env_reference_targets."""
    from duck_gym_b200 import cuda_batch
    from duck_gym_b200.tensor_env import _ptr
    import ctypes

    g = np.load(GOLDEN / "env_gait.npz")
    config = ast.literal_eval(str(g["config"]))
    env = make_env(gait_dir, num_envs=6, task="locomotion", episode_seconds=config["episode_seconds"],
                   action_scale=config["action_scale"], auto_reset=False, gait=True, foot_clearance=True,
                   load_transfer=True)
    np.testing.assert_array_equal(env.gait_table.cpu().numpy(), g["gait_targets"].astype(np.float32))
    lib = cuda_batch.library()
    for i in range(g["actions"].shape[0]):
        cuda_t = lambda name, dtype=torch.float32: torch.from_numpy(np.ascontiguousarray(g[name][i])).cuda().to(dtype)
        a_out, target = torch.empty(6, 14, device="cuda"), torch.empty(6, 14, device="cuda")
        # Inputs bound to names: a temporary's memory could be reused before the launch.
        actions, length, commands = cuda_t("actions"), cuda_t("episode_length", torch.int64), cuda_t("commands")
        cuda_batch._raise(lib.duck_env_reference_targets(
            env.native._h, ctypes.byref(env._params), _ptr(actions), float(config["action_scale"]),
            _ptr(env.home), _ptr(env.lower), _ptr(env.upper), _ptr(length), _ptr(commands), _ptr(a_out),
            _ptr(target), env._stream))
        np.testing.assert_allclose(target.cpu().numpy(), g["applied_targets"][i], rtol=0, atol=1e-6)


@pytest.mark.parametrize("case", ["env_standing", "env_locomotion"])
def test_fused_post_step_on_reference_states(biped_dir, biped_meta, case):
    """The reference env's recorded physics states, loaded into the GPU batch,
    give the reference's recorded masks bit for bit and its observations and
    rewards within tolerance."""
    from duck_gym_b200 import cuda_batch
    from duck_gym_b200.tensor_env import _ptr
    import ctypes

    g = np.load(GOLDEN / f"{case}.npz")
    config = ast.literal_eval(str(g["config"]))
    assert json.loads(str(g["metadata"]))["home"] == biped_meta["home"]
    env = make_env(biped_dir, num_envs=6, task=config["task"], episode_seconds=config["episode_seconds"],
                   velocity_filter_seconds=config["velocity_filter_seconds"], action_scale=config["action_scale"],
                   auto_reset=False)
    lib, h = cuda_batch.library(), env.native._h
    n = 6
    for i in range(g["actions"].shape[0]):
        env.native.import_records(torch.from_numpy(
            records_from_golden(g["bodies"][i], g["diag"][i], env.native.record_length)).cuda())
        def cuda_t(name, dtype=torch.float32):
            return torch.from_numpy(np.ascontiguousarray(g[name][i])).cuda().to(dtype)

        a = cuda_t("actions").clamp(-1, 1).contiguous()
        prev = cuda_t("prev_actions").contiguous()
        length = cuda_t("episode_length", torch.int64).contiguous()
        returns = cuda_t("returns", torch.float32).contiguous()
        commands = cuda_t("commands").contiguous()
        filtered = cuda_t("filtered").contiguous()
        obs = torch.empty(n, env.num_obs, device="cuda")
        reward = torch.empty(n, device="cuda")
        failed, timeout, done = (torch.empty(n, device="cuda", dtype=torch.bool) for _ in range(3))
        cuda_batch._raise(lib.duck_env_post_step(
            h, ctypes.byref(env._params), _ptr(env.home), _ptr(a), _ptr(prev), _ptr(length), _ptr(returns),
            _ptr(commands), _ptr(filtered), _ptr(obs), _ptr(reward), _ptr(failed), _ptr(timeout), _ptr(done),
            None, None, env._stream))
        np.testing.assert_array_equal(failed.cpu().numpy(), g["failed"][i], err_msg=f"{case} step {i}")
        np.testing.assert_array_equal(timeout.cpu().numpy(), g["timeouts"][i])
        np.testing.assert_array_equal(done.cpu().numpy(), g["done"][i])
        np.testing.assert_array_equal(length.cpu().numpy(), g["episode_length"][i] + 1)
        np.testing.assert_allclose(obs.cpu().numpy(), g["terminal_obs"][i], **OBS_TOL)
        np.testing.assert_allclose(reward.cpu().numpy(), g["reward"][i], **REWARD_TOL)


def test_reset_draws_match_reference_generator(biped_dir):
    """Reset noise comes from the reference's generator calls in the
    reference's order: the joint angles after the first reset are home plus
    the first uniform draw of a generator seeded like the env's."""
    env = make_env(biped_dir, num_envs=32, seed=123, task="locomotion")
    gen = torch.Generator(device="cuda").manual_seed(123)
    q = env.home + (torch.rand((32, env.num_actions), generator=gen, device="cuda") - 0.5) * 0.02
    torch.rand((32, 2), generator=gen, device="cuda")
    selected = torch.randint(4, (32,), generator=gen, device="cuda")
    joints = env.native.state()[1][:, :, 0]
    torch.testing.assert_close(joints, q, rtol=0, atol=2e-5)
    want = env._directions[selected] * env.command_speed
    assert torch.equal(env.commands, want)


def test_auto_reset_isolation_and_timeouts(biped_dir):
    env = make_env(biped_dir, num_envs=16, episode_seconds=0.1)   # 5 control steps
    zeros = torch.zeros(16, env.num_actions, device="cuda")
    for step in range(1, 6):
        obs, reward, done, info = env.step(zeros)
        if step < 5:
            assert not info["time_outs"].any()
            assert torch.equal(env.episode_length_buf, torch.full_like(env.episode_length_buf, step))
    # Standing still from home: every env times out together at step 5 ...
    assert info["time_outs"].all() and not info["failed"].any()
    # ... is reset (fresh counters), and the terminal observation is the
    # pre-reset one, not the returned post-reset observation.
    assert (env.episode_length_buf == 0).all() and (env.returns == 0).all()
    assert not torch.equal(info["terminal_observation"], obs)
    assert torch.isfinite(obs).all() and obs.shape == (16, env.num_obs)


def test_failed_env_does_not_disturb_neighbours(biped_dir):
    env = make_env(biped_dir, num_envs=8, auto_reset=False, randomize=False)
    quiet = torch.zeros(8, env.num_actions, device="cuda")
    forces = torch.zeros(8, 3, device="cuda")
    forces[3, 2] = 3 * env.meta["mass"] * 9.81       # lift env 3 off its feet
    env.forces.copy_(forces)
    base = make_env(biped_dir, num_envs=8, auto_reset=False, randomize=False)
    for _ in range(10):
        o1, r1, d1, i1 = env.step(quiet)
        o2, r2, d2, i2 = base.step(quiet)
    assert i1["failed"][3] and not i2["failed"][3]
    keep = torch.arange(8, device="cuda") != 3
    assert torch.equal(i1["terminal_observation"][keep], i2["terminal_observation"][keep])
    assert torch.equal(r1[keep], r2[keep])
