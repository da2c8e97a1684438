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
def model_dir():
    """Where the seeded synthetic model files live: $S2D_MODEL_CACHE, else
    the shared cache of synth.default_model_dir() (RAM-backed when it has
    room), so that the full-size models are written once per host and shared
    with bench.py.  Files are written under a temporary name and renamed."""
    from fish_s2pro_b200 import synth
    d = synth.default_model_dir()
    d.mkdir(parents=True, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def tiny_gguf(model_dir):
    from fish_s2pro_b200 import configs, synth
    return synth.cached_gguf(configs.C1.model, model_dir)


@pytest.fixture(scope="session")
def codec_gguf(model_dir):
    """The seeded synthetic codec file (decode tensors of the real shapes)."""
    from fish_s2pro_b200 import codec_synth
    return codec_synth.cached_codec_gguf(model_dir)


@pytest.fixture(scope="session")
def codec_oracle_weights(codec_gguf):
    from oracle import codec_oracle
    return codec_oracle.CodecWeights(codec_gguf)
