import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def model_dirs(tmp_path_factory):
    from oracle import synth

    base = Path(os.environ.get("QTTS_TEST_MODELS", str(tmp_path_factory.mktemp("models"))))
    return {s: synth.write_model(base / s, s, 0) for s in ("tiny", "tiny_proj")}


@pytest.fixture(scope="session")
def oracles(model_dirs):
    from oracle import qtts_oracle as O

    return {s: O.OracleModel(d, 128) for s, d in model_dirs.items()}


@pytest.fixture(scope="session")
def full_model_dir(tmp_path_factory):
    """Lazily written full-size synthetic checkpoints ("0.6b", "1.7b"), shared
    by every test of the session."""
    from oracle import synth

    base = Path(os.environ.get("QTTS_TEST_MODELS", str(tmp_path_factory.mktemp("full"))))
    made = {}

    def get(shape):
        if shape not in made:
            made[shape] = synth.write_model(base / shape, shape, 0)
        return made[shape]

    return get
