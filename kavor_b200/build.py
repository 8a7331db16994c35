"""Build the sm_100a kernel library ``kavor_b200/libkavor_b200.so`` in tree.

Every ``csrc/*.cu`` is compiled separately with nvcc for ``sm_100a`` and linked
into one shared library that exports the C ABI of ``include/kavor_b200.h``.
The build is incremental (an object is rebuilt when its source or any header
is newer) and runs the compilations in parallel. No GPU is needed.

    python -m kavor_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ = ROOT / "_build" / "obj"
LIB = PKG / "libkavor_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
    "-DKVB_BUILD",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the kavor_b200 kernels need the CUDA toolkit to build")
    return path


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(src: Path, obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, extra: list[str], verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile all kernels and link the shared library; returns its path."""
    OBJ.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    deps = _headers()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    jobs = []
    objs = []
    for src in srcs:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(src, obj, deps):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), max(1, os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(workers) as ex:
            for obj, log in ex.map(lambda j: _compile(j[0], j[1], extra, verbose), jobs):
                if ptxas_verbose and log:
                    print(f"== {obj.stem}\n{log}")
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers / spills / smem per kernel")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
