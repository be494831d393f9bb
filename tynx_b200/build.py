"""Build ``tynx_b200/_lib/libtynx_cuda.so`` with nvcc for sm_100a.

Usage: ``python -m tynx_b200.build [--force] [--jobs N]``.  Objects are rebuilt
when their source or any header under ``csrc/`` / ``include/`` is newer.  The
library is built in-tree so that it travels with the repository.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "_lib"
LIB = OUT / "libtynx_cuda.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-DTYNX_BUILD", "-I", str(INCLUDE),
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    paths = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), "-x", "cu", *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")


def build(force: bool = False, jobs: int = 0, verbose: bool = False, extra: list[str] | None = None) -> Path:
    OUT.mkdir(exist_ok=True)
    objdir = OUT / "obj"
    objdir.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    jobs = jobs or min(len(todo), os.cpu_count() or 4) or 1
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        futures = [pool.submit(_compile, s, o, extra or []) for s, o in todo]
        for f in futures:
            f.result()
    if todo or force or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lnccl", "-lcudart_static",
               "-ldl", "-lrt", "-lpthread"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"built {LIB}")
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=0)
    parser.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v resource usage")
    args = parser.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    if args.ptxas_info:
        for src in sources():
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", os.devnull]
            if src.suffix == ".cpp":
                continue
            result = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(result.stderr)
        return
    build(force=args.force, jobs=args.jobs, verbose=True)


if __name__ == "__main__":
    main()
