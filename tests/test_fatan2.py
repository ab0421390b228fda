"""CPU: the solver's atan2 (csrc/dmath.cuh ``fatan2``) restated in float32
numpy -- the ratio of the smaller to the larger magnitude, the fitted odd
polynomial, the octant and quadrant restored -- against the float64 arctan2
over all four quadrants, both axes and the origin.  The coefficients are read
from the CUDA source, so the test follows any refit."""

import re
from pathlib import Path

import numpy as np

DMATH = Path(__file__).resolve().parents[1] / "duck_gym_b200" / "csrc" / "dmath.cuh"


def coefficients():
    body = DMATH.read_text().split("__device__ __forceinline__ float fatan2(float y, float x) {")[1].split("}")[0]
    first = re.search(r"float p = (-?0x[0-9a-fp.+-]+)f;", body).group(1)
    rest = re.findall(r"p = p \* s ([+-]) (0x[0-9a-fp.+-]+)f;", body)
    values = [float.fromhex(first)] + [float.fromhex(v) * (1 if sign == "+" else -1) for sign, v in rest]
    return np.array(values, np.float32)   # highest degree first


def fatan2(y, x):
    y, x = np.float32(y), np.float32(x)
    ax, ay = np.abs(x), np.abs(y)
    mx, mn = np.maximum(ax, ay), np.minimum(ax, ay)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.where(mx > 0, mn * (np.float32(1) / np.where(mx > 0, mx, 1)), np.float32(0)).astype(np.float32)
    s = t * t
    c = coefficients()
    p = np.full_like(t, c[0])
    for k in c[1:]:
        p = (p * s + k).astype(np.float32)
    p = (p * t).astype(np.float32)
    p = np.where(ay > ax, np.float32(np.pi / 2) - p, p)
    p = np.where(x < 0, np.float32(np.pi) - p, p)
    return np.copysign(p, y)


def test_coefficients_are_eight():
    assert coefficients().size == 8


def test_fatan2_error_over_all_quadrants():
    rng = np.random.default_rng(0)
    angle = rng.uniform(-np.pi, np.pi, 400000)
    radius = np.exp(rng.uniform(-12, 4, angle.size))
    y, x = (radius * np.sin(angle)).astype(np.float32), (radius * np.cos(angle)).astype(np.float32)
    got = fatan2(y, x).astype(np.float64)
    want = np.arctan2(y.astype(np.float64), x.astype(np.float64))
    err = np.abs(got - want)
    assert err.max() < 5e-7, err.max()
    # small angles (rotation logarithms): relative accuracy
    t = np.float32(10.0) ** rng.uniform(-7, -1, 10000).astype(np.float32)
    rel = np.abs(fatan2(t, np.ones_like(t)) - np.arctan2(t.astype(np.float64), 1.0)) / t
    assert rel.max() < 3e-7, rel.max()


def test_fatan2_axes_and_origin():
    for y, x, want in ((0.0, 1.0, 0.0), (1.0, 0.0, np.pi / 2), (0.0, -1.0, np.pi), (-1.0, 0.0, -np.pi / 2),
                       (0.0, 0.0, 0.0), (-0.0, -1.0, -np.pi), (1.0, 1.0, np.pi / 4), (-1.0, -1.0, -3 * np.pi / 4)):
        assert abs(float(fatan2(y, x)) - want) < 5e-7, (y, x)
