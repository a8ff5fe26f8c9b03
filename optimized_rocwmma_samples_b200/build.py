"""Builds libb2sq.so (the C-ABI library) in-tree with nvcc for sm_100a only.

    python -m optimized_rocwmma_samples_b200.build [--force]

Each ``csrc/*.cu`` is compiled to ``_build/*.o`` (in parallel) and linked
with the CUDA runtime statically, so the library does not depend on which
libcudart a host process (e.g. PyTorch) loaded first.  No fast-math: the
smoothquant arithmetic must round exactly like the CPU reference.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libb2sq.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-diag-suppress", "186",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: libb2sq needs the CUDA 12.9 toolkit to build")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + [PKG / "samples" / "b2sq_samples.cpp"] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links libb2sq.so if any source is newer; returns its path."""
    deps = _deps()
    if not force and not _stale(LIB, deps):
        return LIB
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-Xlinker", "--no-undefined", "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of libb2sq.so failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    build_samples(verbose)
    return LIB


SAMPLES_SRC = PKG / "samples" / "b2sq_samples.cpp"
SAMPLES_BIN = PKG / "b2sq_samples"


def build_samples(verbose: bool = False) -> Path:
    """The C++ host driver mirroring the reference samples (links libb2sq.so)."""
    cmd = [nvcc(), *ARCH, "-O2", "-std=c++17", f"-I{INCLUDE}", "-o", str(SAMPLES_BIN), str(SAMPLES_SRC),
           f"-L{PKG}", "-lb2sq", "-Xlinker", "-rpath=$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build of b2sq_samples failed:\n{res.stdout}\n{res.stderr}")
    return SAMPLES_BIN


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
