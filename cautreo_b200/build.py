"""Build libcautreo_b200.so in place: CUDA kernels for sm_100a (nvcc) and the
C11 host layer (gcc), linked into one shared library with the CUDA runtime
linked statically.

    python -m cautreo_b200.build [--force] [--ptxas-verbose]

Object files go to cautreo_b200/_build/; the library lands next to this file
so it travels with the source tree.
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
BUILD = PKG / "_build"
LIB = PKG / "libcautreo_b200.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
CC = shutil.which("gcc") or "gcc"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"), "-I", str(PKG / "csrc"),
]
CC_FLAGS = ["-O2", "-std=c11", "-D_GNU_SOURCE", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter",
            "-I", str(ROOT / "include"), "-I", str(CUDA_HOME / "include")]


def _sources():
    cu = sorted((PKG / "csrc").glob("*.cu"))
    c = sorted((PKG / "host").glob("*.c"))
    headers = sorted((PKG / "csrc").glob("*.h")) + sorted((PKG / "csrc").glob("*.cuh")) + sorted(
        (ROOT / "include").glob("*.h"))
    return cu, c, headers


def _stale(obj: Path, src: Path, headers) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every kernel and host source; return the library path."""
    BUILD.mkdir(exist_ok=True)
    cu, c, headers = _sources()
    jobs_list = []
    for src in cu:
        obj = BUILD / (src.stem + ".cu.o")
        if force or ptxas_verbose or _stale(obj, src, headers):
            flags = NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])
            jobs_list.append((src, [NVCC] + flags + ["-c", str(src), "-o", str(obj)]))
    for src in c:
        obj = BUILD / (src.stem + ".c.o")
        if force or _stale(obj, src, headers):
            jobs_list.append((src, [CC] + CC_FLAGS + ["-c", str(src), "-o", str(obj)]))
    logs = {}
    if jobs_list:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_run, cmd): src for src, cmd in jobs_list}
            for f in cf.as_completed(futs):
                logs[futs[f].name] = f.result()
    objs = [str(BUILD / (s.stem + ".cu.o")) for s in cu] + [str(BUILD / (s.stem + ".c.o")) for s in c]
    if jobs_list or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + objs + ["-lpthread", "-ldl", "-lrt"])
        os.replace(tmp, LIB)
    if ptxas_verbose:
        (BUILD / "ptxas.log").write_text("".join(f"== {k}\n{v}\n" for k, v in sorted(logs.items())))
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, ptxas_verbose=a.ptxas_verbose)
    print(lib)
    if a.ptxas_verbose:
        print((BUILD / "ptxas.log").read_text())


if __name__ == "__main__":
    sys.exit(main())
