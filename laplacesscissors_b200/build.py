"""Builds liblsx.so (the CUDA sm_100a kernels and the C ABI of include/lsx.h) in-tree.

Usage: python laplacesscissors_b200/build.py [--force] [--jobs N]

Each csrc/*.cu compiles to _build/<name>.o with nvcc for sm_100a only; the objects
link into laplacesscissors_b200/liblsx.so.  A source is rebuilt when it or any
header is newer than its object.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "liblsx.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def host_compiler() -> list[str]:
    # The system g++ carries libgomp; prefer it over toolchains that do not.
    for candidate in ("/usr/bin/g++",):
        if Path(candidate).exists():
            return ["-ccbin", candidate]
    return []


def common_flags() -> list[str]:
    return ARCH + host_compiler() + [
        "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-fopenmp,-Wall,-Wno-unused-function,-ffp-contract=off",
        "-I", str(INCLUDE), "-I", str(CSRC),
    ]


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def compile_one(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *common_flags(), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    deps = headers()
    todo = [s for s in sources if force or stale(BUILD / (s.stem + ".o"), s, deps)]
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
            list(pool.map(lambda s: compile_one(s, verbose), todo))
    objects = [BUILD / (s.stem + ".o") for s in sources]
    if force or todo or not LIBRARY.exists() or any(o.stat().st_mtime > LIBRARY.stat().st_mtime for o in objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, *host_compiler(), "-shared", "-o", str(tmp), *map(str, objects),
               "-Xcompiler", "-fopenmp", "-lgomp"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        shutil.move(str(tmp), str(LIBRARY))
    return LIBRARY


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
