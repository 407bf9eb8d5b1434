"""Builds the native library libridge_b200.so in-tree (ridge_b200/lib/).

Every CUDA source is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`), in parallel, then linked with
g++-compatible host objects into one shared library that exports the C ABI
declared in include/ridge_b200.h. Object files go to ridge_b200/_build/ and are
rebuilt only when a source or header is newer than the object.

Usage: python ridge_b200/build.py [-j N] [--verbose] [--ptxas-info]
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
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libridge_b200.so"
CLI = LIBDIR / "ridge-predict"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_HOME = Path(NVCC).resolve().parent.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(ROOT / "include"),
]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-I", str(CSRC), "-I", str(ROOT / "include"),
             "-I", str(CUDA_HOME / "include")]


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(p for p in CSRC.glob("*.cpp") if p.name != "ridge_predict_cli.cpp")
    return cu, cpp


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, headers) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(map(str, cmd)), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    out = (r.stdout or "") + (r.stderr or "")
    if r.returncode != 0:
        raise RuntimeError("command failed:\n%s\n%s" % (" ".join(map(str, cmd)), out))
    return out


def build(jobs: int | None = None, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    cu, cpp = _sources()
    headers = _headers()
    tasks = []
    objs = []
    for src in cu:
        obj = BUILD / (src.stem + ".cu.o")
        objs.append(obj)
        if ptxas_info or _stale(obj, src, headers):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            tasks.append([NVCC, *CUDA_FLAGS, *extra, "-c", str(src), "-o", str(obj)])
    for src in cpp:
        obj = BUILD / (src.stem + ".cpp.o")
        objs.append(obj)
        if _stale(obj, src, headers):
            tasks.append(["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)])
    jobs = jobs or max(1, os.cpu_count() or 1)
    logs = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for out in ex.map(lambda c: _run(c, verbose), tasks):
            logs.append(out)
    if ptxas_info:
        print("\n".join(logs))
    if tasks or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs),
              "-L", str(CUDA_HOME / "lib64"), "-lcudart", "-lpthread", "-ldl"], verbose)
        os.replace(tmp, LIB)
    cli_src = CSRC / "ridge_predict_cli.cpp"
    if cli_src.exists() and (not CLI.exists() or CLI.stat().st_mtime < LIB.stat().st_mtime
                             or cli_src.stat().st_mtime > CLI.stat().st_mtime):
        _run(["g++", *CXX_FLAGS, str(cli_src), "-o", str(CLI), "-L", str(LIBDIR),
              "-lridge_b200", "-Wl,-rpath,$ORIGIN", "-L", str(CUDA_HOME / "lib64"),
              "-lcudart"], verbose)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args(argv)
    lib = build(a.j, a.verbose, a.ptxas_info)
    print("built", lib)


if __name__ == "__main__":
    sys.exit(main())
