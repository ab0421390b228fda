"""Generates the golden vectors in this folder from the reference's own CPU
solver (``_duck_reference.CpuBatch32/64`` built from the reference sources by
``oracle/build_ref.sh``).

Each ``<case>.npz`` stores the model text, the inputs of every call and the
reference's outputs after every call, so ``tests/test_oracle.py`` can replay
the case on the CPU restatement and demand bit equality.  Run from the repo
root:  python tests/golden/make_golden.py
"""

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import helpers  # noqa: E402
from duck_gym_b200 import biped  # noqa: E402
from oracle.oracle import reference_module  # noqa: E402

OUT = Path(__file__).resolve().parent


def record(ref, model_text, case, fp64, dt, iterations, calls, n, nj, offsets=True):
    """calls: list of ("step", target, forces, substeps, kp, limit) or
    ("motor", motor, forces) or ("reset", mask, q, roots)."""
    dtype = np.float64 if fp64 else np.float32
    path = OUT / f"_{case}.duck"
    path.write_text(model_text)
    try:
        batch = (ref.CpuBatch64 if fp64 else ref.CpuBatch32)(str(path), n, dt, iterations, 1)
        outputs = {k: [] for k in ("bodies", "joints", "diag", "forces", "ground_forces", "counts", "self",
                                   "loads")}
        rng = np.random.default_rng(11)
        load_offsets = []
        kinds = []
        for call in calls:
            kind = call[0]
            kinds.append(kind)
            if kind == "step":
                batch.step(*call[1:])
            elif kind == "motor":
                batch.step_motor(*call[1:])
            else:
                batch.reset(*call[1:])
            b, j, d = batch.state()
            outputs["bodies"].append(b)
            outputs["joints"].append(j)
            outputs["diag"].append(d)
            outputs["forces"].append(batch.contact_forces())
            outputs["ground_forces"].append(batch.contact_forces(True))
            outputs["counts"].append(batch.contact_counts())
            outputs["self"].append(batch.self_contact_stats())
            off = rng.normal(0, 0.01, (n, 3)).astype(dtype)
            load_offsets.append(off)
            outputs["loads"].append(batch.generalized_loads(off))
    finally:
        path.unlink()
    arrays = {k: np.stack(v) for k, v in outputs.items()}
    arrays["load_offsets"] = np.stack(load_offsets)
    arrays["model"] = np.array(model_text)
    arrays["meta"] = np.array([int(fp64), n, nj, iterations], np.int64)
    arrays["dt"] = np.array(dt)
    arrays["kinds"] = np.array(kinds)
    # Inputs, padded per kind.
    arrays["targets"] = np.stack([c[1] if c[0] == "step" else np.zeros((n, nj), dtype) for c in calls])
    arrays["step_forces"] = np.stack([c[2] if c[0] in ("step", "motor") else np.zeros((n, 3), dtype)
                                      for c in calls])
    arrays["substeps"] = np.array([c[3] if c[0] == "step" else 0 for c in calls])
    arrays["kp"] = np.array([c[4] if c[0] == "step" else 0.0 for c in calls])
    arrays["limit"] = np.array([c[5] if c[0] == "step" else 0.0 for c in calls])
    arrays["motor"] = np.stack([c[1] if c[0] == "motor" else np.zeros((n, nj, 3), dtype) for c in calls])
    arrays["mask"] = np.stack([c[1] if c[0] == "reset" else np.zeros(n, bool) for c in calls])
    arrays["q"] = np.stack([c[2] if c[0] == "reset" else np.zeros((n, nj), dtype) for c in calls])
    arrays["roots"] = np.stack([c[3] if c[0] == "reset" else np.zeros((n, 6), dtype) for c in calls])
    np.savez_compressed(OUT / f"{case}.npz", **arrays)
    print(case, {k: v.shape for k, v in arrays.items() if k in ("bodies", "targets")})


def main():
    ref = reference_module()
    if ref is None:
        raise SystemExit("oracle/_ref is not built; run oracle/build_ref.sh first")
    rng = np.random.default_rng(0)

    # Biped, fp32, config-1 style: HOME + N(0, 0.1) targets each control step.
    text, meta = biped.generate(0)
    n, nj = 4, 14
    home = np.asarray(meta["home"], np.float32)
    calls = [("reset", np.ones(n, bool), (home + rng.normal(0, 0.02, (n, nj))).astype(np.float32),
              rng.normal(0, 0.01, (n, 6)).astype(np.float32))]
    for s in range(40):
        calls.append(("step", (home + rng.normal(0, 0.1, (n, nj))).astype(np.float32),
                      rng.normal(0, 0.1, (n, 3)).astype(np.float32), 4, meta["kp"], meta["torque_limit"]))
    bad = (home + rng.normal(0, 0.1, (n, nj))).astype(np.float32)
    bad[2, 3] = np.nan
    calls.append(("step", bad, np.zeros((n, 3), np.float32), 4, meta["kp"], meta["torque_limit"]))
    calls.append(("reset", np.array([False, False, True, False]), np.tile(home, (n, 1)),
                  np.zeros((n, 6), np.float32)))
    for s in range(10):
        motor = np.stack([rng.normal(0, 0.05, (n, nj)), rng.uniform(0, 0.01, (n, nj)),
                          rng.uniform(0, 0.02, (n, nj))], -1).astype(np.float32)
        calls.append(("motor", motor, np.zeros((n, 3), np.float32)))
    record(ref, text, "biped_fp32", False, 0.005, 10, calls, n, nj)

    # Biped, fp64, fixed targets.
    n = 3
    home64 = home.astype(np.float64)
    target = home64 + rng.normal(0, 0.05, (n, nj))
    calls = [("step", target, np.zeros((n, 3)), 4, meta["kp"], meta["torque_limit"]) for _ in range(30)]
    record(ref, text, "biped_fp64", True, 0.005, 10, calls, n, nj)

    # Pendulum with limits, dry friction, damping, armature and ground contact.
    n, nj = 4, 1
    t = np.linspace(-0.9, 0.9, n)[:, None]
    for fp64 in (False, True):
        dtype = np.float64 if fp64 else np.float32
        calls = [("step", t.astype(dtype), np.zeros((n, 3), dtype), 2, 5.0, 1.0) for _ in range(60)]
        record(ref, helpers.PENDULUM, f"pendulum_{'fp64' if fp64 else 'fp32'}", fp64, 0.002, 30, calls, n, nj)

    # Two boxes, one collision pair (MPR), no gravity.
    n, nj = 3, 0
    for fp64 in (False, True):
        dtype = np.float64 if fp64 else np.float32
        f = np.zeros((n, 3), dtype)
        f[1, 0] = 0.5
        calls = [("motor", np.zeros((n, 0, 3), dtype), f) if s % 2 else
                 ("step", np.zeros((n, 0), dtype), f, 2, 0.0, 1.0) for s in range(60)]
        record(ref, helpers.box_pair(), f"box_pair_{'fp64' if fp64 else 'fp32'}", fp64, 0.002, 30, calls, n, nj)


if __name__ == "__main__":
    main()
