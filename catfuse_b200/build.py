"""Build the sm_100a shared library ``libcatfuse_sm100.so`` in-tree.

Every ``csrc/*.cu`` file is compiled by ``nvcc`` for ``sm_100a`` in parallel
and linked into one shared object next to this file, so that the library
travels with the source tree (no JIT cache, no site-packages install).

    python -m catfuse_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_NAME = "libcatfuse_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME
INCLUDE_DIR = PKG_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-DNDEBUG",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          extra: list[str] | None = None) -> Path:
    """Compile and link the library; returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    extra = list(extra or [])
    srcs = _sources()
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    # an object is rebuilt when it is older than its source or any shared header
    hdr = max((p.stat().st_mtime for p in _deps() if p.suffix != ".cu"), default=0.0)
    stale = [s for s, o in zip(srcs, objs)
             if force or extra or not o.exists()
             or o.stat().st_mtime < max(s.stat().st_mtime, hdr)]
    if stale:
        jobs = jobs or min(len(stale), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            list(ex.map(lambda s: _compile(s, extra), stale))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true", help="print register/smem usage")
    ap.add_argument("--define", action="append", default=[],
                    help="extra preprocessor definition NAME[=VALUE] (rebuild with --force)")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    extra += [f"-D{d}" for d in args.define]
    if args.ptxas_verbose:
        BUILD_DIR.mkdir(exist_ok=True)
        for src in _sources():
            obj = BUILD_DIR / (src.stem + ".o")
            cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(res.stderr)
        return 0
    build(force=args.force, jobs=args.jobs, verbose=True, extra=extra)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
