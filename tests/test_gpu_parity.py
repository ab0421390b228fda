"""GPU parity tests: the CUDA library (through its C ABI) against the CPU
oracle, on the same seeded inputs.

Tolerances: contact sets and failure flags bit exact; after one substep
from a common state, body poses within 1e-4 m / rad; velocities within 1e-3
in fp32, up to the reference algorithm's own one-ulp envelope measured on the
same checks (helpers.VelocityStats); 1000-step ensemble statistics within 1 %.
"""

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu

POSE_TOL = 1e-4
VEL_TOL = 1e-3


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from duck_gym_b200 import CudaBatch

    return CudaBatch


def oracle(model, n, dt, iterations, fp64=False, threads=8):
    from oracle.oracle import OracleBatch

    return OracleBatch(model, n, dt, iterations, threads=threads, fp64=fp64)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def host_state(batch):
    return [x.cpu().numpy() for x in batch.state()]


def load_oracle_state(gpu, ora):
    rec = np.stack([ora.export_env(e) for e in range(ora.num_envs)])
    gpu.import_records(dev(rec))


class VelocityStats(helpers.VelocityStats):
    """Velocity differences pooled per test and held to the one-ulp envelope
    of the reference algorithm measured on the same checks (helpers.py); the
    poses likewise, with `pose_tol` and no floor, so with twins that stay
    within it the plain pose bound applies (up to three components)."""

    def __init__(self, tol=VEL_TOL, pose_tol=POSE_TOL):
        super().__init__(tol)
        self.poses = helpers.VelocityStats(pose_tol, floor=0.0)

    def check(self):
        super().check()
        self.poses.check()


def twins_for(model, n, dt, iterations, **kw):
    """One-ulp oracle twins of an oracle batch (helpers.UlpTwins)."""
    return helpers.UlpTwins(lambda: oracle(model, n, dt, iterations, **kw))


def compare_substep(gpu, ora, stats, twin_states=(), diag_tol=1e-4):
    gb, gj, gd = host_state(gpu)
    ob, oj, od = ora.state()
    np.testing.assert_array_equal(gd[:, 5], od[:, 5], err_msg="failure flags differ")
    live = od[:, 5] == 0
    for e in range(ora.num_envs):
        np.testing.assert_array_equal(gpu.contact_keys(e), ora.contact_keys(e),
                                      err_msg=f"contact set of env {e} differs")
    stats.poses.add("body pose", gb[live][..., :7], ob[live][..., :7], [t[0][live][..., :7] for t in twin_states])
    stats.poses.add("joint angle", gj[live][..., 0], oj[live][..., 0], [t[1][live][..., 0] for t in twin_states])
    stats.add("body velocity", gb[live][..., 7:], ob[live][..., 7:], [t[0][live][..., 7:] for t in twin_states])
    stats.add("joint rate", gj[live][..., 1], oj[live][..., 1], [t[1][live][..., 1] for t in twin_states])
    np.testing.assert_array_equal(gd[live][:, 2], od[live][:, 2])
    np.testing.assert_allclose(gd[live][:, [0, 1, 4]], od[live][:, [0, 1, 4]], rtol=0, atol=diag_tol)


def teacher_check(gpu, ora, twins, gpu_step, ora_step, stats, **tol):
    """Load the oracle's exact state into the GPU batch (and perturbed copies
    into the twins), advance all of them with the same controls, compare."""
    rec = np.stack([ora.export_env(e) for e in range(ora.num_envs)])
    gpu.import_records(dev(rec))
    gpu_step()
    twin_states = twins.advance(rec, ora_step) if twins is not None else ()
    ora_step(ora)
    compare_substep(gpu, ora, stats, twin_states, **tol)


def test_initial_state_matches_oracle(cuda, biped_model, biped_meta):
    n = 8
    gpu = cuda(biped_model, n, 0.005, 10)
    ora = oracle(biped_model, n, 0.005, 10)
    gb, gj, gd = host_state(gpu)
    ob, oj, od = ora.state()
    np.testing.assert_array_equal(gb, ob)  # copied model state
    np.testing.assert_allclose(gj, oj, rtol=0, atol=1e-6)  # atan2 differs by ulps
    np.testing.assert_array_equal(gd, od)
    q = helpers.home_q(biped_meta, n, noise=0.05)
    roots = np.random.default_rng(2).normal(0, 0.01, (n, 6)).astype(np.float32)
    mask = np.ones(n, bool)
    mask[3] = False
    gpu.reset(dev(mask), dev(q), dev(roots))
    ora.reset(mask, q, roots)
    gb, gj, gd = host_state(gpu)
    ob, oj, od = ora.state()
    np.testing.assert_allclose(gb, ob, rtol=0, atol=2e-6)
    np.testing.assert_allclose(gj, oj, rtol=0, atol=2e-6)
    np.testing.assert_array_equal(gd, od)


@pytest.mark.parametrize("noise,fixed", [(0.1, False), (0.05, True)])
def test_single_substep_teacher_forced(cuda, biped_model, biped_meta, noise, fixed):
    """Along an oracle trajectory, load the oracle's exact state into the GPU
    batch, advance both one substep with the same controls, and compare."""
    n, steps = 16, 60
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    gpu = cuda(biped_model, n, 0.005, 10)
    ora = oracle(biped_model, n, 0.005, 10)
    t = helpers.targets(biped_meta, steps, n, noise, seed=3, fixed=fixed)
    forces = np.random.default_rng(4).normal(0, 0.2, (steps, n, 3)).astype(np.float32)
    q = helpers.home_q(biped_meta, n, noise=0.02)
    roots = np.zeros((n, 6), np.float32)
    ora.reset(np.ones(n, bool), q, roots)
    checked = 0
    stats = VelocityStats()
    twins = twins_for(biped_model, n, 0.005, 10)
    for s in range(steps):
        for sub in range(4):
            if (4 * s + sub) % 7 == 0:
                teacher_check(gpu, ora, twins, lambda: gpu.step(dev(t[s]), dev(forces[s]), 1, kp, limit),
                              lambda b: b.step(t[s], forces[s], 1, kp, limit), stats)
                checked += 1
            else:
                ora.step(t[s], forces[s], 1, kp, limit)
    stats.check()
    contacts = ora.state()[2][:, 2]
    assert checked > 30 and contacts.max() > 0


def test_full_control_step_teacher_forced(cuda, biped_model, biped_meta):
    """A 4-substep call from a common state stays within a few pose tolerances."""
    n, steps = 16, 40
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    gpu = cuda(biped_model, n, 0.005, 10)
    ora = oracle(biped_model, n, 0.005, 10)
    t = helpers.targets(biped_meta, steps, n, 0.05, seed=5, fixed=True)
    f = np.zeros((n, 3), np.float32)
    for s in range(steps):
        if s % 10 == 9:
            load_oracle_state(gpu, ora)
            gpu.step(dev(t[s]), dev(f), 4, kp, limit)
            ora.step(t[s], f, 4, kp, limit)
            gb, _, gd = host_state(gpu)
            ob, _, od = ora.state()
            np.testing.assert_array_equal(gd[:, 5], od[:, 5])
            np.testing.assert_allclose(gb[..., :7], ob[..., :7], rtol=0, atol=5e-4)
        else:
            ora.step(t[s], f, 4, kp, limit)


def run_ensemble(batch, step, state, targets, kp, limit, forces):
    heights, joint_rms, contacts = [], [], []
    for s in range(targets.shape[0]):
        step(targets[s], forces, kp, limit)
        b, j, d = state()
        heights.append(b[:, 1, 2].mean())
        joint_rms.append(np.sqrt(np.mean(j[:, :, 0] ** 2)))
        contacts.append(d[:, 2].mean())
    return np.mean(heights), np.mean(joint_rms), np.mean(contacts)


def test_ensemble_statistics_1000_steps(cuda, biped_model, biped_meta):
    """1000 control steps from HOME with fixed noisy PD targets (the bench
    workload): mean base height, joint RMS and contact count within 1 %."""
    n, steps = 256, 1000
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    t = helpers.targets(biped_meta, 1, n, 0.05, seed=6, fixed=True)[0]
    forces = np.zeros((n, 3), np.float32)
    ora = oracle(biped_model, n, 0.005, 10)
    gpu = cuda(biped_model, n, 0.005, 10)
    tg, fg = dev(t), dev(forces)
    stats = {"oracle": [], "gpu": []}
    for s in range(steps):
        ora.step(t, forces, 4, kp, limit)
        gpu.step(tg, fg, 4, kp, limit)
        for name, st in (("oracle", ora.state()), ("gpu", host_state(gpu))):
            b, j, d = st
            stats[name].append((b[:, 1, 2].mean(), np.sqrt(np.mean(j[:, :, 0] ** 2)), d[:, 2].mean()))
    o = np.mean(stats["oracle"], axis=0)
    g = np.mean(stats["gpu"], axis=0)
    np.testing.assert_allclose(g, o, rtol=0.01)


def test_boundary_contract(cuda, biped_model, biped_meta):
    """The reference's CUDA boundary checks (tests/cuda_boundary.py:1-66)."""
    n = 4
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    e = cuda(biped_model, n, 0.005, 10)
    home = torch.tensor(biped_meta["home"], device="cuda")
    e.reset(torch.ones(n, dtype=torch.bool, device="cuda"), home.repeat(n, 1).contiguous(),
            torch.zeros(n, 6, device="cuda"))
    initial = e.state()[0].clone()
    assert e.contact_forces().abs().sum() == 0
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        target = home.repeat(n, 1)
        target[1, 0] += 0.03
        forces = torch.zeros(n, 3, device="cuda")
        forces[1, 0] = 0.02
        e.step(target, forces, 5, kp, limit)
        del target, forces
    snapshot = e.contact_forces()
    assert torch.isfinite(snapshot).all() and (snapshot[:, :, 2] >= -1e-6).all()
    snapshot.fill_(999)
    assert not (e.contact_forces() == 999).all()
    before = e.state()[0]
    e.reset(torch.tensor([True, False, False, False], device="cuda"), home.repeat(n, 1).contiguous(),
            torch.zeros(n, 6, device="cuda"))
    after = e.state()[0]
    torch.testing.assert_close(after[0], initial[0], rtol=0, atol=1e-7)
    torch.testing.assert_close(after[1:], before[1:], rtol=0, atol=0)
    forces = torch.zeros(n, 3, device="cuda")
    for bad in (home.repeat(n, 1).double(), home.repeat(n, 1)[:, :-1].contiguous(), home.repeat(n, 1).cpu()):
        with pytest.raises(RuntimeError):
            e.step(bad, forces, 1, kp, limit)
    with pytest.raises(RuntimeError):
        e.step(home.repeat(n, 1), forces, 0, kp, limit)
    with pytest.raises(RuntimeError):
        e.step(home.repeat(n, 1), forces, 1, -1.0, limit)
    bad = home.repeat(n, 1)
    bad[2, 0] = float("nan")
    e.step(bad, forces, 1, kp, limit)
    assert e.state()[2][:, 5].tolist() == [0, 0, 1, 0]
    e.reset(torch.tensor([False, False, True, False], device="cuda"), home.repeat(n, 1).contiguous(),
            torch.zeros(n, 6, device="cuda"))
    assert e.state()[2][:, 5].tolist() == [0, 0, 0, 0]
    # Batch-size invariance: env 2 of a batch of 4 equals a single-env batch.
    single = cuda(biped_model, 1, 0.005, 10)
    e.reset(torch.ones(n, dtype=torch.bool, device="cuda"), home.repeat(n, 1).contiguous(),
            torch.zeros(n, 6, device="cuda"))
    single.reset(torch.ones(1, dtype=torch.bool, device="cuda"), home[None].contiguous(),
                 torch.zeros(1, 6, device="cuda"))
    target = home.repeat(n, 1)
    target[:, 0] += 0.03
    forces = torch.tensor([[0.02, 0, 0]], device="cuda").repeat(n, 1)
    e.step(target, forces, 20, kp, limit)
    single.step(target[:1].contiguous(), forces[:1].contiguous(), 20, kp, limit)
    for one, batch in zip(single.state(), e.state()):
        torch.testing.assert_close(one[0], batch[2], rtol=0, atol=0)


def test_step_motor_and_loads_parity(cuda, biped_model, biped_meta):
    n, steps = 8, 30
    gpu = cuda(biped_model, n, 0.005, 10)
    ora = oracle(biped_model, n, 0.005, 10)
    rng = np.random.default_rng(7)
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    t = helpers.targets(biped_meta, steps, n, 0.05, seed=8)
    zero = np.zeros((n, 3), np.float32)
    stats = VelocityStats()
    twins = twins_for(biped_model, n, 0.005, 10)
    for s in range(steps):
        ora.step(t[s], zero, 4, kp, limit)
        if s % 5 == 4:
            load_oracle_state(gpu, ora)
            offset = rng.normal(0, 0.01, (n, 3)).astype(np.float32)
            np.testing.assert_allclose(gpu.generalized_loads(dev(offset)).cpu().numpy(),
                                       ora.generalized_loads(offset), rtol=1e-3, atol=2e-4)
            np.testing.assert_allclose(gpu.contact_forces().cpu().numpy(), ora.contact_forces(), rtol=0, atol=1e-5)
            np.testing.assert_allclose(gpu.contact_forces(True).cpu().numpy(), ora.contact_forces(True),
                                       rtol=0, atol=1e-5)
            np.testing.assert_array_equal(gpu.contact_counts().cpu().numpy(), ora.contact_counts())
            motor = np.stack([rng.normal(0, 0.05, (n, 14)), rng.uniform(0, 0.01, (n, 14)),
                              rng.uniform(0, 0.02, (n, 14))], -1).astype(np.float32)
            motor[1, 3, 1] = -1.0  # invalid friction budget: env 1 fails
            teacher_check(gpu, ora, twins, lambda: gpu.step_motor(dev(motor), dev(zero)),
                          lambda b: b.step_motor(motor, zero), stats)
            ora.reset(np.eye(n, dtype=bool)[1], helpers.home_q(biped_meta, n), np.zeros((n, 6), np.float32))
    stats.check()


def test_fp64_single_substep(cuda, biped_model, biped_meta):
    n, steps = 8, 30
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    gpu = cuda(biped_model, n, 0.005, 10, fp64=True)
    ora = oracle(biped_model, n, 0.005, 10, fp64=True)
    t = helpers.targets(biped_meta, steps, n, 0.1, seed=9).astype(np.float64)
    f = np.zeros((n, 3))
    stats = VelocityStats(tol=1e-6, pose_tol=1e-8)
    twins = twins_for(biped_model, n, 0.005, 10, fp64=True)
    for s in range(steps):
        if s % 6 == 5:
            teacher_check(gpu, ora, twins, lambda: gpu.step(dev(t[s]), dev(f), 1, kp, limit),
                          lambda b: b.step(t[s], f, 1, kp, limit), stats, diag_tol=1e-8)
        ora.step(t[s], f, 4, kp, limit)
    stats.check()


@pytest.mark.parametrize("gap,vx", [(-0.002, 0.2), (0.001, 0.5)])
def test_self_contact_pairs(cuda, tmp_path, gap, vx):
    model = helpers.write(tmp_path, "pair.duck", helpers.box_pair(gap, vx))
    n = 3
    gpu = cuda(model, n, 0.002, 30)
    ora = oracle(model, n, 0.002, 30)
    motor = np.zeros((n, 0, 3), np.float32)
    f = np.zeros((n, 3), np.float32)
    f[1, 0] = 0.5
    seen = 0
    stats = VelocityStats()
    twins = twins_for(model, n, 0.002, 30)
    for s in range(60):
        teacher_check(gpu, ora, twins, lambda: gpu.step_motor(dev(motor), dev(f)),
                      lambda b: b.step_motor(motor, f), stats)
        seen += int(ora.contact_counts()[:, 1].sum())
    stats.check()
    np.testing.assert_allclose(gpu.self_contact_stats().cpu().numpy(), ora.self_contact_stats(), rtol=0,
                               atol=1e-5)
    assert seen > 0


def test_pendulum_limits_friction_ground(cuda, tmp_path):
    model = helpers.write(tmp_path, "pendulum.duck", helpers.PENDULUM)
    n = 4
    gpu = cuda(model, n, 0.002, 30)
    ora = oracle(model, n, 0.002, 30)
    t = np.linspace(-0.9, 0.9, n, dtype=np.float32)[:, None]
    f = np.zeros((n, 3), np.float32)
    stats = VelocityStats()
    twins = twins_for(model, n, 0.002, 30)
    for s in range(80):
        teacher_check(gpu, ora, twins, lambda: gpu.step(dev(t), dev(f), 1, 5.0, 1.0),
                      lambda b: b.step(t, f, 1, 5.0, 1.0), stats)
    stats.check()
    assert ora.state()[2][:, 2].max() > 0


def test_free_body_force_units(cuda, tmp_path):
    """1 kg free body: +9.81 N cancels gravity exactly (reference
    tests/test_python.py:70-84, restated on the CUDA batch)."""
    model = helpers.write(tmp_path, "free.duck", helpers.FREE_BODY)
    b = cuda(model, 2, 0.001, 200)
    f = torch.tensor([[0, 0, 9.81], [1, 0, 9.81]], device="cuda")
    b.step(torch.zeros(2, 0, device="cuda"), f, 100, 0.0, 1.0)
    s = b.state()[0].cpu().numpy()
    np.testing.assert_allclose(s[:, 1, 2], 1, atol=1e-6)
    assert abs(s[1, 1, 0] - 0.00505) < 1e-6
    assert abs(s[1, 1, 7] - 0.1) < 1e-5


def test_reference_method_matches_oracle(cuda, biped_model, biped_meta):
    b = cuda(biped_model, 2, 0.005, 10)
    target = torch.tensor(biped_meta["home"], dtype=torch.float32)
    target[0] += 0.05
    forces = torch.tensor([0.01, 0.0, 0.0])
    gb, gj, gd = [x.numpy() for x in b.reference(target, forces, 3, 20.0, 2.0)]
    ora = oracle(biped_model, 1, 0.005, 10)
    ora.step(target.numpy()[None], forces.numpy()[None], 3, 20.0, 2.0)
    ob, oj, od = ora.state()
    np.testing.assert_allclose(gb, ob[0], rtol=0, atol=5e-4)
    np.testing.assert_array_equal(gd[5], od[0, 5])
