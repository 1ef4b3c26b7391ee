"""Stage the reference implementation itself next to the oracle (TEST / BASELINE INFRASTRUCTURE).

    python oracle/build_ref.py --reference <reference checkout>

The reference's rollout engine is pure Python (PyTorch, plus Triton and FlashAttention on its CUDA
path), so "building" it is making its package importable where the benchmark runs: this copies the
``src/climbing_gym`` package of a reference checkout, unmodified, into ``oracle/_ref/climbing_gym``.
``oracle/_ref/`` is ignored by git (no reference source enters this repository's history) but travels
with the working tree, like the built CUDA library. A manifest with the SHA-256 of every staged file
is written beside it.

Who may import ``oracle/_ref``: ``bench.py --impl reference`` (the reference's own CPU engine timed on
the host cores; with ``--reference-device cuda`` its Triton / FlashAttention / CUDA-graph engine on the
GPU, the comparator named by the rollout target) and tests that check the drop-in boundary against
the reference's engine object. Nothing under ``climbing_gym_b200/`` imports it.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
STAGED = HERE / "_ref"
PACKAGE = "climbing_gym"


def build(reference: str | Path) -> Path | None:
    """Copy the reference package; returns the staged directory, or None when ``reference`` has no
    ``src/climbing_gym`` (e.g. on a machine without the checkout: an earlier staging is left alone)."""
    source = Path(reference) / "src" / PACKAGE
    if not source.is_dir():
        return None
    target = STAGED / PACKAGE
    if target.exists():
        shutil.rmtree(target)
    STAGED.mkdir(parents=True, exist_ok=True)
    shutil.copytree(source, target, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    manifest = {str(path.relative_to(STAGED)): hashlib.sha256(path.read_bytes()).hexdigest()
                for path in sorted(target.rglob("*")) if path.is_file()}
    (STAGED / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return target


def staged_path() -> Path | None:
    """Directory to put on sys.path to import the staged reference, or None when it is not staged."""
    return STAGED if (STAGED / PACKAGE / "inference" / "lfm25_engine.py").exists() else None


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True, help="root of a reference checkout (the directory holding src/)")
    args = parser.parse_args()
    staged = build(args.reference)
    if staged is None:
        sys.exit(f"{args.reference}/src/{PACKAGE} not found")
    print(staged)
