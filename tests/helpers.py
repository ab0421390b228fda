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
