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


def synthetic_tokenizer_json(path):
    """A tokenizer.json of the reference's shape for the tests: the 256
    byte-level symbols (ids 0..255 in byte order), a few merges, and the
    special tokens build_prompt needs, all below the tiny models' 4096 text ids
    (<|im_end|> = 4000, the tiny models' end id)."""
    import json
    from fish_s2pro_b200.text import bytes_to_unicode
    table = bytes_to_unicode()
    vocab = {table[b]: b for b in range(256)}
    sp = chr(0x120)  # the byte-level space
    merges = [("h", "e"), ("l", "l"), ("he", "ll"), (sp, "w"), ("o", "r"), (sp + "w", "or")]
    for i, (a, b) in enumerate(merges):
        vocab[a + b] = 256 + i
    added = [{"id": 3000, "content": "<|im_start|>", "special": True},
             {"id": 4000, "content": "<|im_end|>", "special": True},
             {"id": 3001, "content": "<|voice|>", "special": True},
             {"id": 3002, "content": "<|speaker:0|>", "special": True},
             {"id": 3003, "content": "plain", "special": False}]
    doc = {"added_tokens": added, "model": {"type": "BPE", "vocab": vocab,
                                            "merges": [f"{a} {b}" for a, b in merges]}}
    path.write_text(json.dumps(doc))
    return path


@pytest.fixture(scope="session")
def tokenizer_json(tmp_path_factory):
    return synthetic_tokenizer_json(tmp_path_factory.mktemp("tok") / "tokenizer.json")
