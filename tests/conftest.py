import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("S2D_MODEL_CACHE")
    if d:
        Path(d).mkdir(parents=True, exist_ok=True)
        return Path(d)
    return tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def tiny_gguf(model_dir):
    from fish_s2pro_b200 import configs, synth
    return synth.cached_gguf(configs.C1.model, model_dir)
