"""GPU test of duck_batch_reference_static, the allocation-free entry point.

Some callers cannot call cudaMalloc when they want a single-environment check
of the solver: a host framework whose caching allocator owns the device memory
and forbids raw allocation beside it, a process held to a fixed device-memory
budget, and real-time control loops that must not take the implicit
synchronisation of cudaMalloc/cudaFree.  For them the library keeps this entry
point's scratch in a fixed 32 KiB device array instead of allocating it.  The
test calls it through the C ABI and checks its outputs against
duck_batch_reference (which allocates its scratch) on two calls in a row, on a
batch with per-environment masses, inertias and frictions installed, then
checks that a model too large for the fixed array is rejected with a clear
error.  It lives in a file of its own that pytest
collects last, and passes alone in a fresh process as well as after the rest
of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

POSE_TOL = 1e-4


def bind():
    from duck_gym_b200.cuda_batch import library

    lib = library()
    P, I, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
    for name in ("duck_batch_reference", "duck_batch_reference_static"):
        fn = getattr(lib, name)
        fn.argtypes = [P, P, P, I, D, D, P, P, P]
        fn.restype = I
    lib.duck_last_error.restype = ctypes.c_char_p
    return lib


def call(lib, name, batch, target, forces, substeps, kp, limit):
    dtype = np.float64 if batch.dtype == torch.float64 else np.float32
    bodies = np.full((batch.num_bodies, 13), np.nan, dtype)
    joints = np.full((batch.num_joints, 2), np.nan, dtype)
    diag = np.full(6, np.nan, dtype)
    target = np.ascontiguousarray(target, dtype)
    forces = np.ascontiguousarray(forces, dtype)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    status = getattr(lib, name)(batch._h, ptr(target), ptr(forces), int(substeps), float(kp), float(limit),
                                ptr(bodies), ptr(joints), ptr(diag))
    return status, (bodies, joints, diag)


@pytest.mark.parametrize("fp64", [False, True])
def test_static_reference_matches_allocating_reference(biped_model, biped_meta, fp64):
    from duck_gym_b200 import CudaBatch

    lib = bind()
    batch = CudaBatch(biped_model, 4, 0.005, 10, 0, fp64)
    home = np.asarray(biped_meta["home"])
    rng = np.random.default_rng(31)
    calls = [(home + rng.normal(0, 0.05, home.size), rng.normal(0, 0.05, 3), 3),
             (home + rng.normal(0, 0.1, home.size), np.zeros(3), 5)]
    for target, forces, substeps in calls:  # two calls in a row share the static array
        s1, ref = call(lib, "duck_batch_reference", batch, target, forces, substeps, 20.0, 2.0)
        s2, out = call(lib, "duck_batch_reference_static", batch, target, forces, substeps, 20.0, 2.0)
        assert s1 == 0, lib.duck_last_error()
        assert s2 == 0, lib.duck_last_error()
        for a, b in zip(out, ref):
            assert np.isfinite(a).all()
            np.testing.assert_allclose(a, b, rtol=0, atol=POSE_TOL)
        assert out[2][5] == 0 and out[2][2] == ref[2][2]


def test_static_reference_uses_per_env_parameters(biped_model, biped_meta):
    """With per-environment parameters installed both entry points run
    environment 0's values, and those values change the result."""
    from duck_gym_b200 import CudaBatch

    lib = bind()
    batch = CudaBatch(biped_model, 4, 0.005, 10)
    home = np.asarray(biped_meta["home"])
    rng = np.random.default_rng(32)
    target, forces = home + rng.normal(0, 0.05, home.size), np.zeros(3)
    _, plain = call(lib, "duck_batch_reference", batch, target, forces, 8, 20.0, 2.0)
    nb, ns = batch.num_bodies, batch.num_shapes
    lines = [line for line in open(biped_model).read().splitlines() if line.strip()]
    mass0 = np.array([float(lines[2 + b].split()[1]) for b in range(nb)], np.float32)
    inertia0 = np.array([[float(v) for v in lines[2 + b].split()[2:5]] for b in range(nb)], np.float32)
    scale = rng.uniform(1.3, 1.6, (4, nb)).astype(np.float32)
    dev = lambda a: torch.as_tensor(a, device="cuda").contiguous()
    batch.set_parameters(dev(mass0[None] * scale), dev(inertia0[None] * scale[..., None]),
                         dev(np.full((4, ns), 0.4, np.float32)))
    for _ in range(2):
        before = batch.launches
        s1, ref = call(lib, "duck_batch_reference", batch, target, forces, 8, 20.0, 2.0)
        middle = batch.launches
        s2, out = call(lib, "duck_batch_reference_static", batch, target, forces, 8, 20.0, 2.0)
        assert s1 == 0 and s2 == 0, lib.duck_last_error()
        assert batch.launches - middle == middle - before  # both count their launches
        for a, b in zip(out, ref):
            np.testing.assert_allclose(a, b, rtol=0, atol=POSE_TOL)
    assert np.abs(ref[0] - plain[0]).max() > 10 * POSE_TOL  # the parameters took effect


def chain_model(links=31):
    """A hinged chain of `links` boxes held above the ground: its fp64 record
    (41 KiB) exceeds the static scratch."""
    lines = [f"DUCK_MODEL 1 {links + 1} {links - 1} {links}", "0 0 -9.81 1",
             "world 0 0 0 0 0 0 0 1 0 0 0 0 0 0 0 0 0"]
    for i in range(links):
        lines.append(f"l{i} 0.05 1e-5 1e-5 1e-5 {0.02 * i} 0 0.5 1 0 0 0 0 0 0 0 0 0")
    for i in range(1, links):
        lines.append(f"j{i} {i} {i + 1} 0.01 0 0 -0.01 0 0 0 1 0 0 1 0 1 0 0 1 0 0 0 0 0 0.01 0 0 0 0 0 0")
    for i in range(links):
        lines.append(f"{i + 1} 1 0 0 0 1 0 0 0 0.005 0.005 0.005 0.8 0")
    return "\n".join(lines) + "\n"


def test_static_reference_rejects_oversized_model(tmp_path):
    from duck_gym_b200 import CudaBatch

    lib = bind()
    path = tmp_path / "chain.duck"
    path.write_text(chain_model())
    batch = CudaBatch(path, 2, 0.002, 5, 0, True)
    status, _ = call(lib, "duck_batch_reference_static", batch, np.zeros(batch.num_joints), np.zeros(3), 1, 1.0, 1.0)
    assert status != 0
    message = lib.duck_last_error().decode()
    assert "too large for the static reference scratch" in message and "32768" in message
    # The allocating entry point still serves this model.
    status, out = call(lib, "duck_batch_reference", batch, np.zeros(batch.num_joints), np.zeros(3), 1, 1.0, 1.0)
    assert status == 0 and np.isfinite(out[0]).all()
