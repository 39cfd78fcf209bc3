"""Builds ``bunsen_b200/libgdr.so`` from ``bunsen_b200/csrc`` with nvcc, for
sm_100a only. The library is written in-tree next to this file; objects go to
``bunsen_b200/_build``.

    python -m bunsen_b200.build [--force]
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libgdr.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", "-Xptxas", "-v"]


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def nvcc() -> str:
    cand = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _newest_header() -> float:
    return max(p.stat().st_mtime for p in headers())


def _compile(src: pathlib.Path, force: bool) -> tuple[pathlib.Path, str]:
    obj = OBJ / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime > max(src.stat().st_mtime,
                                                                _newest_header()):
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", "-I", str(ROOT / "include"), "-I", str(CSRC),
           "-o", str(obj), str(src)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}{res.stderr}")
    return obj, res.stdout + res.stderr


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compiles every CUDA source (in parallel) and links one shared library.
    A no-op when the library is newer than every source and header."""
    srcs = sources()
    if (not force and LIB.exists()
            and LIB.stat().st_mtime > max(max(p.stat().st_mtime for p in srcs), _newest_header())):
        return LIB
    OBJ.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as pool:
        results = list(pool.map(lambda s: _compile(s, force), srcs))
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *(str(o) for o, _ in results)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stdout}{res.stderr}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-q" not in sys.argv)
