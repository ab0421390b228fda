"""CPU: the exact squared threshold of the ground-pick separation test.

The reference keeps a new ground pick only 5 mm or more (laterally) from the
earlier ones: ``std::hypot(dx, dy) < .005`` on floats, compared in double
(src/cuda/kernel.cuh:355).  The CUDA kernel decides it as
``dx*dx + dy*dy < kPickApart2`` in double (exact squares, one rounding) --
no square root.  This test derives the constant again by bisection over the
doubles and checks the two decisions agree on seeded samples around the
boundary, with IEEE round-to-nearest arithmetic (numpy), the same the CUDA
``__dmul_rn``/``__dadd_rn`` intrinsics and the host's correctly rounded
``hypotf`` use.
"""

import math
import re
import struct
from pathlib import Path

import numpy as np

SOLVER = Path(__file__).resolve().parents[1] / "duck_gym_b200" / "csrc" / "solver.cuh"


def reference_close(dx, dy):
    """float hypot (correctly rounded: the exact root of the exact double sum
    of squares, rounded once to float) compared with .005 in double."""
    s = float(np.float64(dx) * np.float64(dx) + np.float64(dy) * np.float64(dy))
    return float(np.float32(math.sqrt(s))) < 0.005


def derive():
    d2i = lambda d: struct.unpack("<q", struct.pack("<d", d))[0]
    i2d = lambda i: struct.unpack("<d", struct.pack("<q", i))[0]
    pred = lambda s: float(np.float32(math.sqrt(s))) < 0.005
    lo, hi = d2i(0.0), d2i(1.0)
    while hi - lo > 1:
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if pred(i2d(mid)) else (lo, mid)
    return i2d(hi)


def kernel_constant():
    text = SOLVER.read_text()
    literal = re.search(r"kPickApart2\s*=\s*(0x[0-9a-fp.+-]+);", text).group(1)
    return float.fromhex(literal)


def test_constant_is_the_derived_threshold():
    assert kernel_constant() == derive()


def test_squared_test_matches_hypot_near_the_boundary():
    S = kernel_constant()
    rng = np.random.default_rng(0)
    angle = rng.uniform(0, 2 * np.pi, 200000)
    radius = 0.005 * (1 + rng.uniform(-3e-7, 3e-7, angle.size))
    dx = (radius * np.cos(angle)).astype(np.float32)
    dy = (radius * np.sin(angle)).astype(np.float32)
    close = np.float64(dx) * np.float64(dx) + np.float64(dy) * np.float64(dy) < S
    ref = np.array([reference_close(a, b) for a, b in zip(dx, dy)])
    assert np.array_equal(close, ref)
    assert 0.2 < close.mean() < 0.8   # the samples straddle the boundary
