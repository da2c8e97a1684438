"""Host-side checks of bench.py (no GPU): the CPU reference arm runs on the
single-process stand-in for the process group, prints one complete JSON
line, and maps no library of the package (only oracle/ builds)."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

_RUN = """
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--workload", "C1", "--steps", "2", "--warmup", "1"]
import bench
bench.main()
maps = open("/proc/self/maps").read()
print(json.dumps(sorted({l.split()[-1] for l in maps.splitlines() if l.endswith(".so")
                         and "/repo/" in l})))
"""


def test_single_has_what_the_reference_arm_reads():
    sys.path.insert(0, str(ROOT))
    import bench
    s = bench._Single()
    for attr in ("world", "rank", "local", "barrier", "max", "sum"):
        assert hasattr(s, attr), attr
    assert (s.world, s.rank, s.local) == (1, 0, 0)


def test_reference_arm_line_and_libraries(tmp_path):
    env = dict(os.environ, S2D_MODEL_CACHE=str(tmp_path), OMP_NUM_THREADS="2")
    proc = subprocess.run([sys.executable, "-c", _RUN], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    libs = json.loads(proc.stdout.splitlines()[-1])
    assert libs, "the oracle library should be mapped"
    assert all("/oracle/" in p for p in libs), libs
