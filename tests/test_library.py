"""CPU checks of the C ABI library and the synthetic model generator (no
compute calls: these run without a GPU)."""

import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "duck_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(duck_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from duck_gym_b200 import build

    lib = ctypes.CDLL(str(build.build_library()))
    names = declared_functions()
    assert len(names) >= 18
    for name in names:
        assert hasattr(lib, name), name


def declared_arity():
    """Parameter count of every function declared in the header."""
    text = (ROOT / "include" / "duck_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(duck_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_python_binding_matches_declared_signatures():
    from duck_gym_b200 import cuda_batch

    lib = cuda_batch.library()
    arity = declared_arity()
    bound = [n for n in arity if getattr(lib, n).argtypes is not None]
    assert len(bound) >= 20
    for name in bound:
        assert len(getattr(lib, name).argtypes) == arity[name], name


def test_library_has_no_torch_dependency():
    from duck_gym_b200 import build

    data = build.LIB_PATH.read_bytes()
    assert b"libtorch" not in data and b"libc10" not in data


def test_cuda_batch_fails_loudly_without_a_device(biped_model):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    from duck_gym_b200 import CudaBatch

    with pytest.raises(RuntimeError):
        CudaBatch(biped_model, 4, 0.005, 10)


def test_build_shim_returns_cuda_batch():
    from duck_gym_b200 import CudaBatch, build_cuda

    assert build_cuda.build().CudaBatch is CudaBatch


def test_biped_generator_is_deterministic_and_matches_spec(tmp_path):
    from duck_gym_b200 import biped

    a, meta = biped.generate(0)
    b, _ = biped.generate(0)
    c, _ = biped.generate(1)
    assert a == b and a != c
    header = a.splitlines()[0].split()
    assert header == ["DUCK_MODEL", "1", "16", "14", "15"]
    assert meta["joint_names"] == list(biped.JOINT_NAMES)
    assert abs(meta["mass"] - 0.7) < 1e-9
    lines = a.splitlines()
    links = [float(line.split()[1]) for line in lines[4:18]]
    assert abs(sum(links) - 0.5) < 1e-9
    pairs_text, _ = biped.generate(0, self_contacts=True)
    count = int(pairs_text.splitlines()[2 + 16 + 14 + 15])
    assert count == 15 * 14 // 2 - 14  # all pairs of the 15 bodies but parent-child


def test_biped_loads_in_oracle_with_expected_topology(biped_model, biped_meta):
    from oracle.oracle import OracleBatch

    o = OracleBatch(biped_model, 2, 0.005, 10)
    assert (o.num_bodies, o.num_joints, o.contact_bound) == (16, 14, 60)
    b, j, d = o.state()
    np.testing.assert_allclose(j[0, :, 0], biped_meta["home"], atol=1e-6)
    assert abs(b[0, 1, 2] - biped_meta["root_height"]) < 1e-6
