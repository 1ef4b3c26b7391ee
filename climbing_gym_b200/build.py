"""In-tree nvcc build of libcgym_b200.so for sm_100a.

``python -m climbing_gym_b200.build`` (or ``__graft_entry__.build()``) compiles every ``.cu``
under ``csrc/`` with ``-gencode arch=compute_100a,code=sm_100a`` and links them into
``climbing_gym_b200/libcgym_b200.so`` next to the Python package, so the library travels with
the source tree. Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libcgym_b200.so"
BUILD_DIR = PACKAGE / "csrc" / "build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the cgym_b200 CUDA library cannot be built")
    return found


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > stamp for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted((PACKAGE.parent / "include").glob("*.h"))
    jobs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        if force or _stale(obj, [src, *headers]):
            cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)

    def run(cmd):
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        return proc.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for log in pool.map(run, jobs):
            if verbose and log:
                print(log, file=sys.stderr)
    objects = [str(BUILD_DIR / (src.stem + ".o")) for src in sources]
    if force or jobs or _stale(LIBRARY, objects):
        run([nvcc, "-shared", "-o", str(LIBRARY), *objects, "-lcudart"])
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
