"""The C-ABI library builds, loads and exports every declared entry point
(no GPU needed: nothing here launches device work)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "s2d.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(s2d_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from fish_s2pro_b200 import build, s2d
    build.build_runtime()
    lib = ctypes.CDLL(str(s2d.LIB_PATH))
    syms = header_symbols()
    assert len(syms) >= 15
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # the Python mirror binds exactly the declared entry points
    assert sorted(s2d.SIGNATURES) == syms


def test_struct_layouts_match_header():
    from fish_s2pro_b200 import s2d
    text = (ROOT / "include" / "s2d.h").read_text()
    spec = re.search(r"typedef struct S2dGraphSpec \{(.*?)\} S2dGraphSpec;", text, re.S).group(1)
    fields = re.findall(r"\b(\w+)\s*[,;]", re.sub(r"/\*.*?\*/", "", spec, flags=re.S))
    assert [f for f, _ in s2d._Spec._fields_] == [f for f in fields if f not in ("int32_t", "float")]
    assert ctypes.sizeof(s2d._GenParams) == 24
    assert ctypes.sizeof(s2d._Config) == 20


def test_open_reports_missing_file_without_crashing(tmp_path):
    """s2d_open fails cleanly (no GPU needed to reach the error path when the
    device cannot be selected either)."""
    from fish_s2pro_b200 import s2d
    with pytest.raises(s2d.S2dError) as e:
        s2d.SlowArState.open(tmp_path / "missing.gguf", max_seq_len=16)
    assert e.value.code in (-2, -3)


def test_python_mirror_validates_prompt():
    from fish_s2pro_b200 import s2d
    import numpy as np
    t = s2d.PromptTensor(rows=3, cols=2, data=np.array([10, 20, 1, 2, 3, 4], np.uint32))
    assert s2d.transpose_to_time_major(t).tolist() == [10, 1, 3, 20, 2, 4]
    with pytest.raises(s2d.S2dError, match="length mismatch"):
        s2d.transpose_to_time_major(s2d.PromptTensor(rows=3, cols=2, data=np.zeros(5, np.uint32)))


def test_workload_byte_model():
    from fish_s2pro_b200 import configs
    b = configs.weight_bytes_per_frame(configs.C2.model)
    assert b["slow"] == 7_266_631_680
    assert b["lm_head"] == 20_976_640
    assert b["fast"] == 9 * (807_403_520 + 20_971_520)
    assert configs.kv_bytes_per_position(configs.C2.model) == 147_456


def header_param_counts():
    """Parameter count of every s2d_* declaration in include/s2d.h."""
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "s2d.h").read_text(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(s2d_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        p = " ".join(params.split())
        out[name] = 0 if p in ("", "void") else p.count(",") + 1
    return out


def test_python_signatures_match_header_arity():
    """Each ctypes binding passes as many arguments as the C declaration takes."""
    from fish_s2pro_b200 import s2d
    counts = header_param_counts()
    assert sorted(counts) == sorted(s2d.SIGNATURES)
    wrong = {n: (len(s2d.SIGNATURES[n][1]), c) for n, c in counts.items() if len(s2d.SIGNATURES[n][1]) != c}
    assert not wrong, wrong
