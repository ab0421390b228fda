"""GPU: the two declared extensions beyond the reference's envelope, checked
against the CPU oracle restating the same algorithm.

* More than 32 body-collision pairs (all 91 non-adjacent pairs of the
  15-link biped).  The reference loader rejects more than 32
  pairs (solver.cpp:151-152); ``max_pairs`` raises the limit in both this
  library and the oracle.  Contact sets stay bit-exact, poses within 1e-4.
* Per-environment physical parameters (domain randomisation).  The
  reference shares one model across all envs (kernel.cuh:331); here a batch
  with per-env masses, inertias and ground frictions must match, env by env,
  oracle batches built from model files carrying each env's values.
"""

import json

import numpy as np
import pytest
import torch

import helpers
from test_gpu_parity import VelocityStats, dev, teacher_check

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def oracle(model, n, max_pairs=32, **kw):
    from oracle.oracle import OracleBatch

    return OracleBatch(model, n, 0.005, 10, threads=8, max_pairs=max_pairs, **kw)


@pytest.fixture(scope="module")
def pair_biped(tmp_path_factory):
    from duck_gym_b200 import biped

    d = tmp_path_factory.mktemp("pairs")
    path = biped.write(d, seed=0, self_contacts=True)
    return path, json.loads((d / "metadata.json").read_text())


def test_pair_limit_is_the_references_by_default(pair_biped):
    from duck_gym_b200 import CudaBatch

    path, _ = pair_biped
    with pytest.raises(RuntimeError, match="pair count"):
        CudaBatch(str(path), 4, 0.005, 10)
    with pytest.raises(ValueError):
        oracle(path, 4)
    batch = CudaBatch(str(path), 4, 0.005, 10, max_pairs=128)
    assert batch.num_pairs == 91 and batch.contact_bound == 151


def test_91_pair_self_contact_teacher_forced(pair_biped):
    from duck_gym_b200 import CudaBatch

    path, meta = pair_biped
    n, steps = 16, 40
    kp, limit = meta["kp"], meta["torque_limit"]
    gpu = CudaBatch(str(path), n, 0.005, 10, max_pairs=128)
    ora = oracle(path, n, max_pairs=128)
    t = helpers.targets(meta, steps, n, 0.6, seed=5)
    forces = np.zeros((n, 3), np.float32)
    ora.reset(np.ones(n, bool), helpers.home_q(meta, n, noise=0.02), np.zeros((n, 6), np.float32))
    stats = VelocityStats()
    twins = helpers.UlpTwins(lambda: oracle(path, n, max_pairs=128))
    checked = self_seen = 0
    for s in range(steps):
        for sub in range(4):
            if (4 * s + sub) % 3 == 0:
                teacher_check(gpu, ora, twins, lambda: gpu.step(dev(t[s]), dev(forces), 1, kp, limit),
                              lambda b: b.step(t[s], forces, 1, kp, limit), stats)
                np.testing.assert_array_equal(gpu.contact_counts().cpu().numpy(), ora.contact_counts())
                checked += 1
            else:
                ora.step(t[s], forces, 1, kp, limit)
            self_seen += int(ora.contact_counts()[:, 1].sum())
    stats.check()
    assert checked > 40 and self_seen > 0


def randomized(meta_model, n, seed):
    """Per-env masses x U[0.8, 1.2] (inertia scaled alike) and ground friction
    U[0.4, 1.2] per env, as float32 arrays."""
    text = meta_model.read_text()
    lines = text.splitlines()
    nb, nj, ns = (int(v) for v in lines[0].split()[2:5])
    mass0 = np.array([float(lines[2 + b].split()[1]) for b in range(nb)], np.float32)
    inertia0 = np.array([[float(v) for v in lines[2 + b].split()[2:5]] for b in range(nb)], np.float32)
    rng = np.random.default_rng(seed)
    scale = rng.uniform(0.8, 1.2, (n, nb)).astype(np.float32)
    mass = (mass0[None] * scale).astype(np.float32)
    inertia = (inertia0[None] * scale[..., None]).astype(np.float32)
    friction = np.repeat(rng.uniform(0.4, 1.2, (n, 1)), ns, axis=1).astype(np.float32)
    return text, mass, inertia, friction


def test_domain_randomization_matches_per_env_models(tmp_path, biped_model, biped_meta):
    from duck_gym_b200 import CudaBatch, biped

    n, steps = 4, 30
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    text, mass, inertia, friction = randomized(biped_model, n, seed=8)
    gpu = CudaBatch(str(biped_model), n, 0.005, 10)
    gpu.set_parameters(dev(mass), dev(inertia), dev(friction))
    oras = []
    for e in range(n):
        path = tmp_path / f"env{e}.duck"
        path.write_text(biped.with_parameters(text, mass[e], inertia[e], friction[e]))
        oras.append(oracle(path, 1))
    t = helpers.targets(biped_meta, steps, n, 0.1, seed=9)
    pushes = np.random.default_rng(10).normal(0, 0.5, (steps, n, 3)).astype(np.float32)
    for e, o in enumerate(oras):
        o.reset(np.ones(1, bool), helpers.home_q(biped_meta, 1, noise=0.02, seed=e), np.zeros((1, 6), np.float32))
    offset = np.zeros((n, 3), np.float32)
    stats = VelocityStats()
    twins = [helpers.UlpTwins(lambda e=e: oracle(tmp_path / f"env{e}.duck", 1)) for e in range(n)]
    for s in range(steps):
        rec = np.concatenate([o.export_env(0)[None] for o in oras])
        gpu.import_records(dev(rec))
        gpu.step(dev(t[s]), dev(pushes[s]), 1, kp, limit)
        twin_states = [tw.advance(rec[e:e + 1], lambda b, e=e: b.step(t[s][e:e + 1], pushes[s][e:e + 1], 1, kp,
                                                                       limit)) for e, tw in enumerate(twins)]
        for e, o in enumerate(oras):
            o.step(t[s][e:e + 1], pushes[s][e:e + 1], 1, kp, limit)
        gb, gj, gd = [x.cpu().numpy() for x in gpu.state()]
        for e, o in enumerate(oras):
            ob, oj, od = o.state()
            assert gd[e, 5] == od[0, 5]
            np.testing.assert_array_equal(gpu.contact_keys(e), o.contact_keys(0), err_msg=f"env {e} step {s}")
            np.testing.assert_allclose(gb[e, :, :7], ob[0, :, :7], rtol=0, atol=1e-4)
            np.testing.assert_allclose(gj[e, :, 0], oj[0, :, 0], rtol=0, atol=1e-4)
            stats.add("body velocity", gb[e, :, 7:], ob[0, :, 7:], [ts[0][0, :, 7:] for ts in twin_states[e]])
            stats.add("joint rate", gj[e, :, 1], oj[0, :, 1], [ts[1][0, :, 1] for ts in twin_states[e]])
        loads = gpu.generalized_loads(dev(offset)).cpu().numpy()
        for e, o in enumerate(oras):
            np.testing.assert_allclose(loads[e], o.generalized_loads(offset[e:e + 1])[0], rtol=1e-3, atol=2e-4)
    stats.check()
    # The envs really differ: the same controls give different trajectories.
    assert np.abs(gb[0, 1, :3] - gb[1, 1, :3]).max() > 1e-6


def test_parameter_validation_and_restore(biped_model, biped_meta):
    from duck_gym_b200 import CudaBatch

    n = 4
    kp, limit = biped_meta["kp"], biped_meta["torque_limit"]
    _, mass, inertia, friction = randomized(biped_model, n, seed=3)
    plain = CudaBatch(str(biped_model), n, 0.005, 10)
    batch = CudaBatch(str(biped_model), n, 0.005, 10)
    bad = mass.copy()
    bad[1, 3] = np.nan
    fr = friction.copy()
    fr[2, 0] = -1
    batch.set_parameters(dev(bad), None, dev(fr))
    diag = batch.state()[2].cpu().numpy()
    assert diag[:, 5].tolist() == [0, 1, 1, 0]
    # Clearing the overrides and resetting gives the shared-model physics back.
    batch.set_parameters(None, None, None)
    mask = torch.ones(n, dtype=torch.bool, device="cuda")
    q = dev(helpers.home_q(biped_meta, n))
    roots = torch.zeros(n, 6, device="cuda")
    for b in (plain, batch):
        b.reset(mask, q, roots)
    target = dev(helpers.targets(biped_meta, 1, n, 0.05, seed=1)[0])
    forces = torch.zeros(n, 3, device="cuda")
    for _ in range(5):
        for b in (plain, batch):
            b.step(target, forces, 4, kp, limit)
    assert torch.equal(plain.state()[0], batch.state()[0])
