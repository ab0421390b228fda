"""Runs a seeded trajectory on the reference's CPU solver rebuilt with a
128-pair capacity (oracle/build_ref_raised.sh) and saves every call's outputs
to an .npz.  Run as a separate process by tests/test_oracle_raised.py: the
rebuilt module registers the same pybind11 types as the unmodified one, so the
two are never loaded into one interpreter.

    python tests/ref_raised_run.py MODEL OUT.npz ENVS STEPS SEED KP LIMIT
"""

import importlib.util
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def module():
    found = sorted((ROOT / "oracle" / "_ref" / "raised").glob("_duck_reference_raised*.so"))
    if not found:
        return None
    spec = importlib.util.spec_from_file_location("_duck_reference_raised", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def trajectory(batch_factory, model, n, steps, seed, kp, limit, home):
    """The inputs both solvers see: HOME + N(0, 0.02) start, HOME + N(0, 0.6)
    targets per step (the legs fold into each other), base forces N(0, 0.2)."""
    rng = np.random.default_rng(seed)
    nj = home.size
    b = batch_factory(model, n)
    q = (home + rng.normal(0, 0.02, (n, nj))).astype(np.float32)
    b.reset(np.ones(n, bool), q, np.zeros((n, 6), np.float32))
    out = {k: [] for k in ("bodies", "joints", "diag", "forces", "counts", "self")}
    for _ in range(steps):
        t = (home + rng.normal(0, 0.6, (n, nj))).astype(np.float32)
        f = rng.normal(0, 0.2, (n, 3)).astype(np.float32)
        b.step(t, f, 4, kp, limit)
        bodies, joints, diag = b.state()
        out["bodies"].append(bodies)
        out["joints"].append(joints)
        out["diag"].append(diag)
        out["forces"].append(b.contact_forces())
        out["counts"].append(b.contact_counts())
        out["self"].append(b.self_contact_stats())
    return {k: np.stack(v) for k, v in out.items()}


if __name__ == "__main__":
    model, out, n, steps, seed, kp, limit = sys.argv[1:8]
    mod = module()
    if mod is None:
        sys.exit("oracle/_ref/raised is not built")
    import json

    home = np.asarray(json.loads((Path(model).parent / "metadata.json").read_text())["home"], np.float32)
    res = trajectory(lambda m, k: mod.CpuBatch32(str(m), k, 0.005, 10, 2), model, int(n), int(steps), int(seed),
                     float(kp), float(limit), home)
    np.savez(out, **res)
