"""Builds the CUDA library ``latent_b200/_lib/liblatent_b200.so`` for sm_100a.

Plain nvcc, in-tree: every translation unit under ``csrc/`` is compiled to an
object in ``_build/`` (in parallel) and linked into one shared library whose
exported symbols are exactly the ``extern "C"`` entry points declared in
``include/latent_ffn.h``.

    python -m latent_b200.build [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
OUT = PKG / "_lib" / "liblatent_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build latent_b200")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _digest(extra_flags) -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + [ROOT / "include" / "latent_ffn.h"]):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS + list(extra_flags)).encode())
    return h.hexdigest()


def build(verbose: bool = False, force: bool = False, extra_flags=()) -> Path:
    stamp = OUT.with_suffix(".sha256")
    digest = _digest(extra_flags)
    if not force and OUT.exists() and stamp.exists() and stamp.read_text() == digest:
        return OUT
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    OUT.parent.mkdir(exist_ok=True)
    ptxas = ["-Xptxas", "-v"] if verbose else []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *extra_flags, *ptxas, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
        if verbose and res.stderr:
            sys.stderr.write(res.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(tmp),
           "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, OUT)
    stamp.write_text(digest)
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
