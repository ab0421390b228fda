"""Shared helpers for the parity tests: seeded inputs and small hand-written
models (the reference's own fixtures need MuJoCo to regenerate, so the cases
below are authored directly in the DUCK_MODEL format)."""

from pathlib import Path

import numpy as np

# A free 1 kg box under gravity (the force-units case of the reference's
# tests/test_python.py:70-84 restated as a model file of our own).
FREE_BODY = """DUCK_MODEL 1 2 0 0
0 0 -9.81 0
world 0 0 0 0 0 0 0 1 0 0 0 0 0 0 0 0 0
base 1 .1 .1 .1 0 0 1 1 0 0 0 0 0 0 0 0 0
"""

# One hinged pendulum link with a limited hinge, a ground plane and a box
# shape: exercises joint rows, limits and ground contact.
PENDULUM = """DUCK_MODEL 1 2 1 1
0 0 -9.81 1
world 0 0 0 0 0 0 0 1 0 0 0 0 0 0 0 0 0
link 0.5 0.002 0.002 0.0003 0.1 0 0.03 1 0 0 0 0 0 0 0 0 0
hinge 0 1 0 0 0.03 -0.1 0 0 0 1 0 0 1 0 1 0 0 1 0 0 1 -0.6 0.6 0.01 0.0002 0.001 0 0 0 0
1 1 0 0 0 1 0 0 0 0.02 0.02 0.02 0.8 0
"""

# Two boxes on two free bodies with one collision pair and no ground: the
# self-contact (MPR) path.  Mirrors the two-body momentum setup of the
# reference's tests/test_body_contacts.py:17-54 with boxes.
def box_pair(gap=-0.002, vx=0.2):
    return f"""DUCK_MODEL 2 3 0 2
0 0 0 0
world 0 0 0 0 0 0 0 1 0 0 0 0 0 0 0 0 0
a 1 0.0004 0.0004 0.0004 {-0.02 - gap / 2} 0 0.1 1 0 0 0 {vx} 0.05 0 0 0 0
b 2 0.0008 0.0008 0.0008 {0.02 + gap / 2} 0.003 0.1 0.9950042 0 0 0.0998334 -0.1 0 0 0 0 0.3
1 1 0 0 0 1 0 0 0 0.02 0.02 0.02 0.5 0 0
2 1 0 0 0 1 0 0 0 0.02 0.02 0.02 0.5 0 0
1
0 1 0.5
"""


def write(tmp_path, name, text):
    path = Path(tmp_path) / name
    path.write_text(text)
    return path


def targets(meta, steps, envs, noise, seed=0, fixed=False):
    """HOME + N(0, noise) joint targets [steps, envs, J] (float32)."""
    rng = np.random.default_rng(seed)
    home = np.asarray(meta["home"], np.float32)
    if fixed:
        t = home + rng.normal(0, noise, (1, envs, home.size))
        return np.repeat(t, steps, axis=0).astype(np.float32)
    return (home + rng.normal(0, noise, (steps, envs, home.size))).astype(np.float32)


def home_q(meta, envs, noise=0.0, seed=1):
    rng = np.random.default_rng(seed)
    home = np.asarray(meta["home"], np.float32)
    return (home + rng.normal(0, noise, (envs, home.size))).astype(np.float32)


# ---------------------------------------------------------------------------
# One-ulp sensitivity of the reference algorithm (the velocity envelope).
#
# Velocities are (x - x0) / h, so at dt = 5 ms they magnify fp32 rounding of
# the poses 200 times, and a stick/slip, limit or friction switch taken the
# other way moves them by much more.  The envelope the GPU is held to is
# measured, not chosen: on every teacher-forced check the CPU oracle (bit for
# bit the reference's own CpuBatch32) also advances copies of the same state
# whose body poses and velocities were moved by one ulp, and the spread of
# those copies around the unperturbed oracle is the reference algorithm's own
# sensitivity to one rounding of its input.

def body_slots(nb):
    """Indices of the body pose/velocity words (x, q, v, w) of bodies 1..B-1
    in a portable record (header 8, then 16 words per body)."""
    idx = [8 + 16 * b + k for b in range(1, nb) for k in range(13)]
    return np.asarray(idx, np.int64)


def perturb_records(records, nb, seed):
    """Copies of `records` [n, L] with every body pose/velocity word moved by
    one ulp, up or down at random (seeded)."""
    out = np.array(records, copy=True)
    idx = body_slots(nb)
    rng = np.random.default_rng(seed)
    up = rng.random((out.shape[0], idx.size)) < 0.5
    vals = out[:, idx]
    out[:, idx] = np.where(up, np.nextafter(vals, np.inf, dtype=out.dtype),
                           np.nextafter(vals, -np.inf, dtype=out.dtype))
    return out


class UlpTwins:
    """Oracle copies advanced from one-ulp-perturbed copies of a state."""

    def __init__(self, make_oracle, seeds=(101, 202, 303)):
        self.seeds = seeds
        self.twins = [make_oracle() for _ in seeds]

    def advance(self, records, step):
        """Load perturbed copies of `records`, apply `step(batch)` to each
        twin, return their states."""
        states = []
        for seed, twin in zip(self.seeds, self.twins):
            rec = perturb_records(records, twin.num_bodies, seed)
            for e in range(twin.num_envs):
                twin.import_env(e, rec[e])
            step(twin)
            states.append(twin.state())
        return states


class VelocityStats:
    """Pools |differences| of one quantity over all checks of one test, for
    the GPU and for the one-ulp twins, and holds the GPU's distribution of
    deviations to the twins' at every level t = tol, 10 tol, 100 tol, ...:

        fraction of GPU components beyond t
            <= 2 x the twins' fraction beyond t (+ `floor` at t = tol)
               + 3 components (sampling noise of the tail).

    With floor = 0 and twins that stay within `tol` this is the plain bound
    `tol` with at most three outliers.
    """

    def __init__(self, tol, floor=1e-3):
        self.tol, self.floor, self.gpu, self.ulp = tol, floor, {}, {}

    def add(self, what, actual, expected, twins=()):
        self.gpu.setdefault(what, []).append(np.abs(actual - expected).ravel())
        for t in twins:
            self.ulp.setdefault(what, []).append(np.abs(t - expected).ravel())

    def check(self):
        for what, parts in self.gpu.items():
            diff = np.concatenate(parts)
            if diff.size == 0:
                continue
            ulp = np.concatenate(self.ulp[what]) if what in self.ulp else np.zeros(1)
            print(f"{what}: GPU {np.mean(diff > self.tol):.6f} beyond {self.tol} (max {diff.max():.3e}); "
                  f"one-ulp twins {np.mean(ulp > self.tol):.6f} (max {ulp.max():.3e}); {diff.size} components")
            level = self.tol
            while True:
                gpu = float(np.mean(diff > level))
                allowed = 2 * float(np.mean(ulp > level)) + (self.floor if level == self.tol else 0.0) \
                    + 3.0 / diff.size
                assert gpu <= allowed, (f"{what}: {gpu:.6f} of components beyond {level:.1e}, "
                                        f"allowed {allowed:.6f} from the one-ulp twins")
                if level >= diff.max():
                    break
                level *= 10


def contact_keys_from_records(records, nb, nj):
    """Per-env (body, shape, feature, other, otherShape) rows read from
    portable records [n, L]: header word 1 is the contact count, contacts
    start after the bodies (16 words each) and joints (22 words each)."""
    base = 8 + 16 * nb + 22 * nj
    out = []
    for rec in np.asarray(records):
        count = int(rec[1])
        rows = rec[base:base + 32 * count].reshape(count, 32)[:, :5]
        out.append(rows.astype(np.int64))
    return out
