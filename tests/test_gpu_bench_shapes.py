"""GPU parity at the launch shapes the benchmark reports, from the states it
times.

* The pure-engine step: 4096 envs (1024 four-env CTAs, the timed launch),
  settled 200 control steps with the benchmark's fixed targets, then
  teacher-forced against the oracle for one substep and for a full 4-substep
  call.
* The self-contact workload: 16384 envs of the 91-pair biped, a few
  substeps teacher-forced against the raised-limit oracle.
* The domain-randomised workload: 65536 envs at 20 iterations with per-env
  parameters, one substep of the whole batch, checked on 32 envs spread over
  it against one-env oracle batches carrying each env's values.
* The CPU-runnable workload as written: 16 envs, 1000 control steps of HOME +
  N(0, 0.1 rad) targets drawn per joint per step, ensemble statistics (mean
  base height, joint RMS, contact count) within 1 % of the oracle's.

Contact sets and failure flags bit exact; poses within 1e-4 and velocities
within 1e-3, each up to the one-ulp envelope of the reference algorithm
measured on the same states (helpers.VelocityStats; with no outlier among
the twins the pose bound is the plain 1e-4).
"""

import json
import os

import numpy as np
import pytest
import torch

import helpers
from test_gpu_parity import VelocityStats, dev

pytestmark = pytest.mark.gpu

THREADS = min(64, os.cpu_count() or 1)
POSE_TOL = 1e-4


def oracle(model, n, iterations=10, **kw):
    from oracle.oracle import OracleBatch

    return OracleBatch(model, n, 0.005, iterations, threads=THREADS, **kw)


def bench_targets(meta, envs):
    """The benchmark's targets: HOME + N(0, 0.05) fixed per env, seed 0."""
    rng = np.random.default_rng(0)
    home = np.asarray(meta["home"], np.float32)
    return (home + rng.normal(0, 0.05, (envs, home.size))).astype(np.float32)


def load(ora, records):
    for e in range(ora.num_envs):
        ora.import_env(e, records[e])


def compare_records(gpu, ora, stats, poses, twin_states=()):
    """Contact sets from the records (one bulk copy), failure flags and
    contact counts exactly; poses and joint angles (`poses`) and velocities
    (`stats`) pooled against the one-ulp twins on the same states."""
    nb, nj = gpu.num_bodies, gpu.num_joints
    grec = gpu.export_records().cpu().numpy()
    orec = np.stack([ora.export_env(e) for e in range(ora.num_envs)])
    gk = helpers.contact_keys_from_records(grec, nb, nj)
    ok = helpers.contact_keys_from_records(orec, nb, nj)
    bad = [e for e in range(len(gk)) if not np.array_equal(gk[e], ok[e])]
    assert not bad, f"contact sets differ in {len(bad)} envs, first {bad[:5]}"
    gb, gj, gd = [x.cpu().numpy() for x in gpu.state()]
    ob, oj, od = ora.state()
    np.testing.assert_array_equal(gd[:, 5], od[:, 5], err_msg="failure flags differ")
    live = od[:, 5] == 0
    np.testing.assert_array_equal(gd[live][:, 2], od[live][:, 2])
    far = np.abs(gb[..., :7] - ob[..., :7]).max(axis=(1, 2))
    worst = int(np.argmax(np.where(live, far, 0)))
    print(f"largest pose deviation {far[worst]:.3e} in env {worst}")
    poses.add("body pose", gb[live][..., :7], ob[live][..., :7], [t[0][live][..., :7] for t in twin_states])
    poses.add("joint angle", gj[live][..., 0], oj[live][..., 0], [t[1][live][..., 0] for t in twin_states])
    stats.add("body velocity", gb[live][..., 7:], ob[live][..., 7:], [t[0][live][..., 7:] for t in twin_states])
    stats.add("joint rate", gj[live][..., 1], oj[live][..., 1], [t[1][live][..., 1] for t in twin_states])
    return int(live.sum())


def test_bench_shape_4096_envs_from_settled_state(biped_model, biped_meta):
    from duck_gym_b200 import CudaBatch

    envs = 4096
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    gpu = CudaBatch(biped_model, envs, 0.005, 10)
    assert (gpu.envs_per_block, gpu.lanes_per_env) == (4, 8)     # 1024 CTAs of 32 lanes, the timed launch
    target = bench_targets(biped_meta, envs)
    tg, fg = dev(target), torch.zeros(envs, 3, device="cuda")
    for _ in range(200):                                          # the benchmark's settle steps
        gpu.step(tg, fg, 4, kp, limit)
    settled = gpu.export_records().cpu().numpy()
    ora = oracle(biped_model, envs)
    twins = helpers.UlpTwins(lambda: oracle(biped_model, envs))
    forces = np.zeros((envs, 3), np.float32)
    stats, poses = VelocityStats(), helpers.VelocityStats(POSE_TOL, floor=0.0)
    # Two substeps teacher-forced from the settled state, then a full call.
    load(ora, settled)
    for _ in range(2):
        rec = np.stack([ora.export_env(e) for e in range(envs)])
        gpu.import_records(dev(rec))
        gpu.step(tg, fg, 1, kp, limit)
        states = twins.advance(rec, lambda b: b.step(target, forces, 1, kp, limit))
        ora.step(target, forces, 1, kp, limit)
        live = compare_records(gpu, ora, stats, poses, states)
    stats.check()
    poses.check()
    assert live >= 0.5 * envs and ora.state()[2][:, 2].mean() > 2   # standing, on its feet
    # A full 4-substep call from the settled state: poses within 5e-4 up to
    # the one-ulp envelope of the same call (four substeps compound it).
    load(ora, settled)
    gpu.import_records(dev(settled))
    gpu.step(tg, fg, 4, kp, limit)
    full = lambda b: b.step(target, forces, 4, kp, limit)
    states = twins.advance(settled, full)
    full(ora)
    gb, _, gd = [x.cpu().numpy() for x in gpu.state()]
    ob, _, od = ora.state()
    np.testing.assert_array_equal(gd[:, 5], od[:, 5])
    live = od[:, 5] == 0
    call = helpers.VelocityStats(5e-4, floor=0.0)
    call.add("body pose (4 substeps)", gb[live][..., :7], ob[live][..., :7], [t[0][live][..., :7] for t in states])
    call.check()


def test_self_contact_16384_envs(tmp_path):
    from duck_gym_b200 import CudaBatch, biped

    path = biped.write(tmp_path, seed=0, self_contacts=True)
    meta = json.loads((tmp_path / "metadata.json").read_text())
    envs = 16384
    kp, limit = meta["kp"], meta["torque_limit"]
    gpu = CudaBatch(str(path), envs, 0.005, 10, max_pairs=128)
    assert gpu.num_pairs == 91
    q = dev(helpers.home_q(meta, envs, noise=0.02))
    gpu.reset(torch.ones(envs, dtype=torch.bool, device="cuda"), q, torch.zeros(envs, 6, device="cuda"))
    t = helpers.targets(meta, 30, envs, 0.6, seed=5)
    fg = torch.zeros(envs, 3, device="cuda")
    for s in range(30):
        gpu.step(dev(t[s]), fg, 4, kp, limit)
    start = gpu.export_records().cpu().numpy()
    ora = oracle(path, envs, max_pairs=128)
    twins = helpers.UlpTwins(lambda: oracle(path, envs, max_pairs=128))
    forces = np.zeros((envs, 3), np.float32)
    stats, poses = VelocityStats(), helpers.VelocityStats(POSE_TOL, floor=0.0)
    load(ora, start)
    target = t[-1]
    self_contacts = 0
    for _ in range(3):
        rec = np.stack([ora.export_env(e) for e in range(envs)])
        gpu.import_records(dev(rec))
        gpu.step(dev(target), fg, 1, kp, limit)
        states = twins.advance(rec, lambda b: b.step(target, forces, 1, kp, limit))
        ora.step(target, forces, 1, kp, limit)
        compare_records(gpu, ora, stats, poses, states)
        np.testing.assert_array_equal(gpu.contact_counts().cpu().numpy(), ora.contact_counts())
        self_contacts += int(ora.contact_counts()[:, 1].sum())
    stats.check()
    poses.check()
    assert self_contacts > 100


def test_cpu_runnable_workload_1000_steps(biped_model, biped_meta):
    """16 envs from HOME, HOME + N(0, 0.1 rad) targets per joint per control
    step, 1000 control steps: ensemble statistics within 1 %."""
    from duck_gym_b200 import CudaBatch

    n, steps = 16, 1000
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    t = helpers.targets(biped_meta, steps, n, 0.1, seed=11)
    forces = np.zeros((n, 3), np.float32)
    q = helpers.home_q(biped_meta, n)
    ora = oracle(biped_model, n)
    gpu = CudaBatch(biped_model, n, 0.005, 10)
    ora.reset(np.ones(n, bool), q, np.zeros((n, 6), np.float32))
    gpu.reset(torch.ones(n, dtype=torch.bool, device="cuda"), dev(q), torch.zeros(n, 6, device="cuda"))
    fg = dev(forces)
    stats = {"oracle": [], "gpu": []}
    for s in range(steps):
        ora.step(t[s], forces, 4, kp, limit)
        gpu.step(dev(t[s]), fg, 4, kp, limit)
        for name, (b, j, d) in (("oracle", ora.state()), ("gpu", [x.cpu().numpy() for x in gpu.state()])):
            stats[name].append((b[:, 1, 2].mean(), np.sqrt(np.mean(j[:, :, 0] ** 2)), d[:, 2].mean()))
    o = np.mean(stats["oracle"], axis=0)
    g = np.mean(stats["gpu"], axis=0)
    print(f"oracle (height, joint RMS, contacts) {o}, GPU {g}")
    np.testing.assert_allclose(g, o, rtol=0.01)


def test_domain_randomized_65536_envs_sample(tmp_path, biped_model, biped_meta):
    """The domain-randomised launch shape: 65536 envs at 20 iterations with
    per-env masses, inertias and ground frictions, joint-offset resets and
    base pushes for 20 control steps; then one substep of the whole batch
    from its own state, checked on 32 envs spread over the batch against
    one-env oracle batches built from model files carrying each env's values."""
    from duck_gym_b200 import CudaBatch, biped
    from test_gpu_extensions import randomized

    envs, sample = 65536, np.linspace(0, 65535, 32).astype(int)
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    text, mass, inertia, friction = randomized(biped_model, envs, seed=21)
    gpu = CudaBatch(str(biped_model), envs, 0.005, 20)
    gpu.set_parameters(dev(mass), dev(inertia), dev(friction))
    q = helpers.home_q(biped_meta, envs, noise=0.02, seed=22)
    gpu.reset(torch.ones(envs, dtype=torch.bool, device="cuda"), dev(q), torch.zeros(envs, 6, device="cuda"))
    target = dev(helpers.targets(biped_meta, 1, envs, 0.05, seed=23)[0])
    rng = np.random.default_rng(24)
    for _ in range(20):
        push = (rng.random((envs, 1)) < 0.02) * rng.normal(0, 0.5, (envs, 3)) * mass[:, 1:2] / (4 * 0.005)
        gpu.step(target, dev(push.astype(np.float32)), 4, kp, limit)
    start = gpu.export_records().cpu().numpy()
    t = target.cpu().numpy()
    zero = torch.zeros(envs, 3, device="cuda")
    gpu.step(target, zero, 1, kp, limit)
    grec = gpu.export_records().cpu().numpy()
    gb, gj, gd = [x.cpu().numpy() for x in gpu.state()]
    stats, poses = VelocityStats(), helpers.VelocityStats(POSE_TOL, floor=0.0)
    nb, nj = gpu.num_bodies, gpu.num_joints
    for e in sample:
        path = tmp_path / f"env{e}.duck"
        path.write_text(biped.with_parameters(text, mass[e], inertia[e], friction[e]))
        make = lambda: oracle(path, 1, iterations=20)
        ora = make()
        ora.import_env(0, start[e])
        twins = helpers.UlpTwins(make)
        step = lambda b: b.step(t[e:e + 1], np.zeros((1, 3), np.float32), 1, kp, limit)
        tw = twins.advance(start[e:e + 1], step)
        step(ora)
        ob, oj, od = ora.state()
        np.testing.assert_array_equal(helpers.contact_keys_from_records(grec[e:e + 1], nb, nj)[0],
                                      helpers.contact_keys_from_records(ora.export_env(0)[None], nb, nj)[0],
                                      err_msg=f"contact set of env {e}")
        assert gd[e, 5] == od[0, 5] and gd[e, 2] == od[0, 2]
        if od[0, 5]:
            continue
        poses.add("body pose", gb[e, :, :7], ob[0, :, :7], [x[0][0, :, :7] for x in tw])
        poses.add("joint angle", gj[e, :, 0], oj[0, :, 0], [x[1][0, :, 0] for x in tw])
        stats.add("body velocity", gb[e, :, 7:], ob[0, :, 7:], [x[0][0, :, 7:] for x in tw])
        stats.add("joint rate", gj[e, :, 1], oj[0, :, 1], [x[1][0, :, 1] for x in tw])
    stats.check()
    poses.check()
    assert np.abs(gb[sample[0], 1, :3] - gb[sample[1], 1, :3]).max() > 1e-6
