"""CPU: the oracle's raised body-pair limit pinned to the reference.

The reference rejects more than 32 body-collision pairs (src/solver.cpp:
151-152, src/cuda/model.hpp:26-29, kernel.cuh:328), so the 91-pair biped can
only be compared with a rebuild of the reference's own CPU solver whose pair
capacity is raised to 128 (oracle/build_ref_raised.sh: four constants changed
in a temporary copy of the sources, a declared deviation).  The restated
oracle with ``max_pairs=128`` must reproduce it bit for bit: states, contact
forces, contact counts and self-contact statistics after every call of a
trajectory in which the legs fold into each other.
"""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import OracleBatch
import ref_raised_run

pytestmark = pytest.mark.skipif(not any((ref_raised_run.ROOT / "oracle" / "_ref" / "raised").glob("*.so")),
                                reason="raised reference not built (oracle/build_ref_raised.sh)")


def test_oracle_bit_exact_with_raised_reference(tmp_path):
    from duck_gym_b200 import biped

    path = biped.write(tmp_path, seed=0, self_contacts=True)
    meta = json.loads((tmp_path / "metadata.json").read_text())
    n, steps, seed = 4, 40, 12
    out = tmp_path / "ref.npz"
    subprocess.run([sys.executable, str(Path(ref_raised_run.__file__)), str(path), str(out), str(n), str(steps),
                    str(seed), str(meta["kp"]), str(meta["torque_limit"])], check=True)
    ref = np.load(out)
    home = np.asarray(meta["home"], np.float32)
    ora = ref_raised_run.trajectory(
        lambda m, k: OracleBatch(m, k, 0.005, 10, threads=2, max_pairs=128, cuda_semantics=False), path, n, steps,
        seed, meta["kp"], meta["torque_limit"], home)
    assert ref["counts"][..., 1].sum() > 0          # body-pair contacts happened
    assert (ref["counts"][..., 1] > 0).any(axis=1).sum() > 3
    for key in ("bodies", "joints", "diag", "forces", "counts", "self"):
        np.testing.assert_array_equal(ora[key], ref[key], err_msg=key)
