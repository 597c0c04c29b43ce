import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("BMO_MODEL_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def tiny_model(model_dir):
    from bmo_jetson_b200 import synth
    return synth.ensure_model("tiny", model_dir)


@pytest.fixture(scope="session")
def tiny17_model(model_dir):
    from bmo_jetson_b200 import synth
    return synth.ensure_model("tiny17", model_dir)
