"""CPU: host-side checks of duck_gym_b200.TensorEnv (argument handling of the
reference's constructor, tensor_env.py:59-176), raised before any device work."""

import pytest

from duck_gym_b200.tensor_env import TensorEnv


@pytest.mark.parametrize("kwargs,error", [
    (dict(substeps=0), ValueError),
    (dict(episode_seconds=0), ValueError),
    (dict(action_scale=0), ValueError),
    (dict(backend="tpu"), ValueError),
    (dict(backend="cpu"), ValueError),
    (dict(gait=True), FileNotFoundError),     # no gait.npz next to the model
])
def test_constructor_rejects(biped_dir, kwargs, error):
    with pytest.raises(error):
        TensorEnv(biped_dir, **kwargs)


def test_params_layout_matches_header():
    import ctypes
    import re
    from pathlib import Path

    from duck_gym_b200.tensor_env import EnvParams

    header = (Path(__file__).resolve().parents[1] / "include" / "duck_b200.h").read_text()
    body = re.search(r"typedef struct duck_env_params \{(.*?)\} duck_env_params;", header, re.S).group(1)
    names = re.findall(r"\b([a-z_]+)(?:\[\d+\])?\s*[,;]", re.sub(r"/\*.*?\*/", "", body, flags=re.S))
    assert [n for n, _ in EnvParams._fields_] == names


def _struct_fields(name):
    import re
    from pathlib import Path

    header = (Path(__file__).resolve().parents[1] / "include" / "duck_b200.h").read_text()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), header, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        names = decl.split(None, 1)[1] if not decl.startswith("const ") else decl.split(None, 2)[2]
        for item in names.split(","):
            fields.append(re.sub(r"[\s*]|\[.*", "", item))
    return fields


def test_bam_structs_match_header():
    import ctypes

    from duck_gym_b200.bam_env import BamBufferTable, BamParams

    assert [n for n, _ in BamParams._fields_] == _struct_fields("duck_bam_params")
    assert [n for n, _ in BamBufferTable._fields_] == _struct_fields("duck_bam_buffers")
    assert ctypes.sizeof(BamBufferTable) == 8 * len(BamBufferTable._fields_)


def test_bam_env_rejects_cpu_backend(tmp_path):
    from duck_gym_b200 import biped
    from duck_gym_b200.bam_env import BamEnv

    biped.write_bam(tmp_path, seed=0)
    with pytest.raises(ValueError):
        BamEnv(tmp_path, backend="cpu")
