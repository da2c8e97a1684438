"""Regenerate the committed golden vectors of the C1 (tiny) workload.

    python tests/golden/make_golden.py

The goldens are outputs of the CPU oracle (oracle/s2_oracle.c, the restatement
of the reference's rust-pure path) on the seeded synthetic C1 model written by
fish_s2pro_b200.synth.  They pin the oracle, the synthetic writer and the
prompt generator across hosts: tests compare fresh oracle and GPU runs against
them.  The reference itself (Rust) cannot be run in this image.
"""
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from fish_s2pro_b200 import configs, synth  # noqa: E402
from oracle import oracle as o  # noqa: E402

OUT = Path(__file__).resolve().parent / "c1_oracle.json"


def make(model_path) -> dict:
    wl = configs.C1
    m = wl.model
    prompt = wl.prompt()
    om = o.OracleModel(model_path, max_seq_len=wl.prompt_len + wl.frames + 8, mode=0)
    flat = prompt.T.reshape(-1).astype(np.int32)
    hidden, logits = om.eval(flat, logits=True)
    sem = logits[m.sem_begin:m.sem_end + 1]
    gp = wl.gen_params(greedy=True)
    codes, mains = om.generate_codes(prompt, gp, o.SeededRng(0))
    gp_s = wl.gen_params(greedy=False)
    gp_s["max_new_tokens"] = 8
    codes_s, mains_s = om.generate_codes(prompt, gp_s, o.SeededRng(1234))
    fast = om.fast_prefix_logits(hidden, [5, 17])
    return {
        "workload": "C1",
        "gguf_sha256": hashlib.sha256(Path(model_path).read_bytes()).hexdigest(),
        "prompt_sha256": hashlib.sha256(prompt.tobytes()).hexdigest(),
        "prefill_hidden_first8": [float(x) for x in hidden[:8]],
        "prefill_semantic_logits_first8": [float(x) for x in sem[:8]],
        "prefill_semantic_argmax": int(np.argmax(sem)),
        "prefill_logits_sha256": hashlib.sha256(logits.tobytes()).hexdigest(),
        "fast_prefix_5_17_first8": [float(x) for x in fast[:8]],
        "greedy_params": gp,
        "greedy_codes": codes.tolist(),
        "greedy_main_tokens": mains.tolist(),
        "sampled_params": gp_s,
        "sampled_seed": 1234,
        "sampled_codes": codes_s.tolist(),
        "sampled_main_tokens": mains_s.tolist(),
    }


if __name__ == "__main__":
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(Path(d) / "c1.gguf", configs.C1.model)
        OUT.write_text(json.dumps(make(path), indent=1) + "\n")
    print(OUT)
