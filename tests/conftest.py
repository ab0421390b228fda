import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs through the C ABI")


@pytest.fixture(scope="session")
def biped_dir(tmp_path_factory):
    from duck_gym_b200 import biped

    d = tmp_path_factory.mktemp("biped")
    biped.write(d, seed=0)
    return d


@pytest.fixture(scope="session")
def biped_model(biped_dir):
    return biped_dir / "microduck.duck"


@pytest.fixture(scope="session")
def biped_meta(biped_dir):
    import json

    return json.loads((biped_dir / "metadata.json").read_text())


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    return oracle.library()
