"""CPU tests of the oracle (the CPU restatement in oracle/): it must reproduce
the reference's own CPU solver bit for bit, on the committed golden vectors
and, where the reference build is present, on fresh random trajectories."""

from pathlib import Path

import numpy as np
import pytest

import helpers
from oracle.oracle import OracleBatch, count_ops, reference_module

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("env_", "bam_")))   # env fixtures


@pytest.mark.parametrize("case", CASES)
def test_oracle_reproduces_golden_vectors(case, tmp_path):
    g = np.load(GOLDEN / f"{case}.npz")
    fp64, n, nj, iterations = (int(v) for v in g["meta"])
    model = helpers.write(tmp_path, "m.duck", str(g["model"]))
    ora = OracleBatch(model, n, float(g["dt"]), iterations, fp64=bool(fp64), cuda_semantics=False)
    for i, kind in enumerate(g["kinds"]):
        if kind == "step":
            ora.step(g["targets"][i], g["step_forces"][i], int(g["substeps"][i]), float(g["kp"][i]),
                     float(g["limit"][i]))
        elif kind == "motor":
            ora.step_motor(g["motor"][i], g["step_forces"][i])
        else:
            ora.reset(g["mask"][i], g["q"][i], g["roots"][i])
        b, j, d = ora.state()
        for name, value in (("bodies", b), ("joints", j), ("diag", d), ("forces", ora.contact_forces()),
                            ("ground_forces", ora.contact_forces(True)), ("counts", ora.contact_counts()),
                            ("self", ora.self_contact_stats()),
                            ("loads", ora.generalized_loads(g["load_offsets"][i]))):
            np.testing.assert_array_equal(value, g[name][i], err_msg=f"{case} call {i} {name}")


def test_golden_cases_exercise_the_paths():
    seen = {}
    for case in CASES:
        g = np.load(GOLDEN / f"{case}.npz")
        seen[case] = (g["counts"][..., 0].max(), g["counts"][..., 1].max(), g["diag"][..., 5].max())
    assert seen["biped_fp32"][0] > 0 and seen["biped_fp32"][2] == 1   # ground contacts, a NaN failure
    assert seen["box_pair_fp32"][1] > 0                                  # body-pair contacts
    assert seen["pendulum_fp32"][0] > 0


REF = reference_module()


@pytest.mark.skipif(REF is None, reason="reference CPU solver not built (oracle/build_ref.sh)")
@pytest.mark.parametrize("fp64", [False, True])
def test_oracle_bit_exact_with_reference_build(fp64, biped_model, biped_meta):
    dtype = np.float64 if fp64 else np.float32
    n, nj = 5, 14
    ref = (REF.CpuBatch64 if fp64 else REF.CpuBatch32)(str(biped_model), n, 0.005, 10, 2)
    ora = OracleBatch(biped_model, n, 0.005, 10, threads=2, fp64=fp64, cuda_semantics=False)
    rng = np.random.default_rng(21)
    home = np.asarray(biped_meta["home"])
    q = (home + rng.normal(0, 0.03, (n, nj))).astype(dtype)
    roots = rng.normal(0, 0.01, (n, 6)).astype(dtype)
    ref.reset(np.ones(n, bool), q, roots)
    ora.reset(np.ones(n, bool), q, roots)
    for s in range(60):
        t = (home + rng.normal(0, 0.15, (n, nj))).astype(dtype)
        f = rng.normal(0, 0.2, (n, 3)).astype(dtype)
        ref.step(t, f, 4, biped_meta["kp"], biped_meta["torque_limit"])
        ora.step(t, f, 4, biped_meta["kp"], biped_meta["torque_limit"])
        for a, b in zip(ref.state(), ora.state()):
            np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(ref.contact_forces(), ora.contact_forces())
    off = rng.normal(0, 0.01, (n, 3)).astype(dtype)
    np.testing.assert_array_equal(ref.generalized_loads(off), ora.generalized_loads(off))


@pytest.mark.skipif(REF is None, reason="reference CPU solver not built (oracle/build_ref.sh)")
def test_convex_narrow_phase_matches_reference_query(tmp_path):
    """Box-box MPR cases of the reference's tests/test_convex.py:20-34, 72-82,
    run through the reference's convex_query32 and through a two-box model on
    the oracle: both find the same contact."""
    box = np.array([[x, y, z] for x in (-1, 1) for y in (-1, 1) for z in (-1, 1)], float) * 0.01
    poses = np.array([[0, 0, 0, 1, 0, 0, 0], [0.019, 0, 0, 1, 0, 0, 0]], float)
    c = REF.convex_query32(box, box, poses)
    assert c["status"] == 1 and abs(c["depth"] - 0.001) < 2e-6
    np.testing.assert_allclose(c["normal"], [-1, 0, 0], atol=1e-6)
    poses[1, 0] = 0.025
    assert REF.convex_query32(box, box, poses)["status"] == 0
    poses[1, 0] = 0.0
    assert abs(REF.convex_query32(box, box, poses)["depth"] - 0.02) < 2e-6


def test_batch_and_thread_invariance(biped_model, biped_meta):
    """Reference tests/test_tensor_env.py:71-96: env results do not depend on
    the batch size or the worker count, bit for bit."""
    n = 3
    a = OracleBatch(biped_model, n, 0.005, 10, threads=1)
    b = OracleBatch(biped_model, n, 0.005, 10, threads=3)
    single = OracleBatch(biped_model, 1, 0.005, 10)
    home = np.asarray(biped_meta["home"], np.float32)
    for step in range(15):
        action = (home + 0.1 * np.sin(np.arange(14) + step * 0.1)).astype(np.float32)
        t = np.tile(action, (n, 1))
        f = np.zeros((n, 3), np.float32)
        a.step(t, f, 4, 20.0, 2.0)
        b.step(t, f, 4, 20.0, 2.0)
        single.step(t[:1], f[:1], 4, 20.0, 2.0)
    for x, y, z in zip(a.state(), b.state(), single.state()):
        np.testing.assert_array_equal(x, y)
        np.testing.assert_array_equal(x[1], z[0])


def test_numeric_failure_isolated_and_resettable(biped_model, biped_meta):
    n = 3
    o = OracleBatch(biped_model, n, 0.005, 10)
    t = np.tile(np.asarray(biped_meta["home"], np.float32), (n, 1))
    t[1, 0] = np.nan
    o.step(t, np.zeros((n, 3), np.float32), 1, 20.0, 2.0)
    assert o.state()[2][:, 5].tolist() == [0, 1, 0]
    o.reset(np.array([False, True, False]), np.zeros((n, 14), np.float32), np.zeros((n, 6), np.float32))
    assert o.state()[2][:, 5].tolist() == [0, 0, 0]
    motor = np.zeros((n, 14, 3), np.float32)
    motor[2, 0, 2] = -1.0
    o.step_motor(motor, np.zeros((n, 3), np.float32))
    assert o.state()[2][:, 5].tolist() == [0, 0, 1]


@pytest.mark.parametrize("text", ["", "DUCK_MODEL 2", "DUCK_MODEL 2 3 0 2\n0 0 0 0\n",
                                  helpers.FREE_BODY + "extra"])
def test_truncated_or_trailing_model_rejected(tmp_path, text):
    path = helpers.write(tmp_path, "broken.duck", text)
    with pytest.raises(ValueError):
        OracleBatch(path, 1, 0.001, 200)


def test_force_units(tmp_path):
    """1 kg free body: +9.81 N cancels gravity (reference tests/test_python.py:70-84)."""
    path = helpers.write(tmp_path, "free.duck", helpers.FREE_BODY)
    o = OracleBatch(path, 2, 0.001, 200, fp64=True)
    o.step(np.zeros((2, 0)), np.array([[0, 0, 9.81], [1, 0, 9.81]]), 100, 0.0, 1.0)
    b = o.state()[0]
    np.testing.assert_allclose(b[:, 1, 2], 1, atol=1e-12)
    assert abs(b[1, 1, 0] - 0.00505) < 1e-10
    assert abs(b[1, 1, 7] - 0.1) < 1e-10


def test_operation_count(biped_model, biped_meta):
    n, steps = 2, 3
    home = np.asarray(biped_meta["home"], np.float32)
    targets = np.tile(home, (steps, n, 1)).astype(np.float32)
    c = count_ops(biped_model, home, targets, np.zeros((n, 3), np.float32), 0.005, 10, 4, 20.0, 2.0)
    assert c["physics_steps"] == steps * n * 4
    per_step = (c["add"] + c["mul"] + c["div"] + c["sqrt"]) / c["physics_steps"]
    assert 1e5 < per_step < 1e7
    assert c["gs_iterations"] <= c["physics_steps"] * 10


def test_operation_count_from_records(biped_model, biped_meta):
    """Counting from exported records continues the HOME run exactly: the
    counts of 3 + 2 steps equal those of 5 steps (the record round trip and
    the counting scalar both reproduce the solver's state bit for bit)."""
    n = 3
    home = np.asarray(biped_meta["home"], np.float32)
    targets = helpers.targets(biped_meta, 5, n, 0.1, seed=4)
    forces = np.zeros((n, 3), np.float32)
    args = (0.005, 10, 4, 20.0, 2.0)
    whole = count_ops(biped_model, home, targets, forces, *args)
    first = count_ops(biped_model, home, targets[:3], forces, *args)
    ora = OracleBatch(biped_model, n, 0.005, 10)
    ora.reset(np.ones(n, bool), np.tile(home, (n, 1)), np.zeros((n, 6), np.float32))
    for s in range(3):
        ora.step(targets[s], forces, 4, 20.0, 2.0)
    records = np.stack([ora.export_env(e) for e in range(n)])
    rest = count_ops(biped_model, home, targets[3:], forces, *args, records=records)
    for key in whole:
        assert whole[key] == first[key] + rest[key], key
