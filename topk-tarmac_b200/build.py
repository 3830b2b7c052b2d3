"""Build the sm_100a shared library libtarmac_b200.so in-tree.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (``-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3``, IEEE division and square
root, no fast-math) into ``_build/*.o`` and links them into
``tarmac_b200/libtarmac_b200.so``. The library exports only the C ABI of
``include/tarmac_b200.h``; the CUDA runtime is linked statically so the
library does not depend on which libcudart the host process loaded.

Usage: ``python topk-tarmac_b200/build.py [--force] [-j JOBS]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "tarmac_b200" / "libtarmac_b200.so"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(INCLUDE),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc",
                 shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to "
                       "build libtarmac_b200.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return (sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh"))
            + sorted(INCLUDE.glob("*.h")))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    hdrs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in [src, *hdrs])


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None,
          extra: list[str] | None = None, verbose: bool = False) -> Path:
    """Compile and link; returns the library path. Rebuilds only stale objects
    unless ``force``."""
    extra = list(extra or [])
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    todo = [s for s in srcs if force or _stale(BUILD / (s.stem + ".o"), s)]
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj in ex.map(lambda s: _compile(s, extra), todo):
                if verbose:
                    print("compiled", obj.name, flush=True)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    newest = max(o.stat().st_mtime for o in objs)
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC",
               "-cudart", "static", *map(str, objs), "-o", str(LIB)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("linked", LIB, flush=True)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print register / spill / shared-memory use")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    if args.ptxas_verbose:
        # -v output goes to stderr of each nvcc call: compile one by one
        BUILD.mkdir(exist_ok=True)
        for s in _sources():
            cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(s), "-o",
                   str(BUILD / (s.stem + ".o"))]
            r = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(r.stderr)
            if r.returncode != 0:
                return r.returncode
    build(force=args.force or args.ptxas_verbose, jobs=args.jobs,
          verbose=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
