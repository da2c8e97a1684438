"""In-tree build of the native libraries.

libs2d.so        the sm_100a Dual-AR runtime (C ABI: include/s2d.h)
libs2d_synth.so  the seeded synthetic GGUF writer (host C)

Both land next to this file so that they travel with the repository to a GPU
host.  `python -m fish_s2pro_b200.build` rebuilds whatever is out of date.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libs2d.so"
SYNTH_LIB = PKG / "libs2d_synth.so"

CUDA_SOURCES = ["s2d_kernels.cu", "s2d_engine.cu", "s2d_prefill.cu", "s2d_decode_attn.cu", "s2d_tcgemm.cu", "s2d_runtime.cu",
                "s2d_gguf.cpp", "s2d_noalloc.cu", "s2d_tc_attn.cu", "s2d_codec.cu",
                "s2d_codec_conv.cu"]
CUDA_HEADERS = ["s2d_common.cuh", "s2d_kernels.cuh", "s2d_sample.cuh", "s2d_prefill.cuh", "s2d_tcgemm.cuh", "s2d_tc_common.cuh",
                "s2d_gguf.h", "s2d_codec.cuh"]
CUDA_LIB = "/usr/local/cuda/lib64"
NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libs2d.so")


def _host_cc() -> str:
    # The system gcc ships libgomp; a relocated gcc earlier on PATH may not.
    return "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_runtime(force: bool = False, verbose_ptxas: bool = False) -> Path:
    deps = [CSRC / s for s in CUDA_SOURCES + CUDA_HEADERS] + [ROOT / "include" / "s2d.h", ROOT / "include" / "s2d_codec.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [
        _nvcc(), *NVCC_ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-shared", "-o", str(LIB),
        *[str(CSRC / s) for s in CUDA_SOURCES],
        f"-L{CUDA_LIB}", "-lcublas", "-ldl", "-Xlinker", f"-rpath={CUDA_LIB}",
    ]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    _run(cmd)
    return LIB


def build_synth(force: bool = False) -> Path:
    src = CSRC / "synth_gguf.c"
    if not force and not _stale(SYNTH_LIB, [src]):
        return SYNTH_LIB
    _run([_host_cc(), "-O3", "-std=gnu11", "-fPIC", "-fopenmp", "-shared", "-o", str(SYNTH_LIB),
          str(src), "-lm"])
    return SYNTH_LIB


def build_oracle(force: bool = False) -> Path:
    """The CPU oracle is test infrastructure; building it is not using it."""
    odir = ROOT / "oracle"
    args = ["make", "-C", str(odir)]
    if force:
        args.insert(1, "-B")
    _run(args)
    return odir / "libs2_oracle.so"


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_oracle(force)
    build_runtime(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(LIB)
