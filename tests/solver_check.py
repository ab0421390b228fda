"""Runs one scene of tests/solver_cases.py through the reference's FP64
solver ``duck_sim`` (oracle/_ref, built by oracle/build_ref.sh) and through a
batch with the CudaBatch interface, and measures the reference's gates
(scripts/validate_cuda.py:77-121): the largest body position and rotation
error against duck_sim, the largest joint error and penetration, checked
every 10 steps as the reference does."""

import subprocess
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
DUCK_SIM = ROOT / "oracle" / "_ref" / "duck_sim"
DT, ITERATIONS = 0.001, 200


def duck_sim(model, steps):
    """Body positions [steps + 1, B - 1, 3] and quaternions [.., 4] of duck_sim."""
    with tempfile.TemporaryDirectory() as d:
        out = Path(d) / "cpu.csv"
        subprocess.run([str(DUCK_SIM), str(model), "--steps", str(steps), "--iterations", str(ITERATIONS),
                        "--output", str(out)], check=True, capture_output=True, text=True)
        rec = np.genfromtxt(out, delimiter=",", names=True)
    nb = int(rec["body"].max())
    pos = np.stack([rec[k] for k in ("x", "y", "z")], -1).reshape(steps + 1, nb, 3)
    quat = np.stack([rec[k] for k in ("qw", "qx", "qy", "qz")], -1).reshape(steps + 1, nb, 4)
    return pos, quat


def measure(batch_step, batch_state, pos, quat, steps):
    """batch_step(n) advances n steps; batch_state() -> (bodies [E,B,13],
    diag [E,6]) as numpy.  Returns the gate quantities."""
    worst = rotation = joint = penetration = 0.0
    for k in range(0, steps, 10):
        n = min(10, steps - k)
        batch_step(n)
        b, diag = batch_state()
        assert not diag[:, 5].any() and np.isfinite(b).all()
        q = b[0, 1:, 3:7].astype(np.float64)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        rotation = max(rotation, float((2 * np.arccos(np.clip(np.abs((q * quat[k + n]).sum(-1)), 0, 1))).max()))
        joint = max(joint, float(diag[:, 0].max()))
        penetration = max(penetration, float(diag[:, 1].max()))
        worst = max(worst, float(np.linalg.norm(b[0, 1:, :3] - pos[k + n], axis=-1).max()))
    return dict(position=worst, rotation=rotation, joint=joint, penetration=penetration)
