"""Build libb2p.so in-tree with nvcc for sm_100a (no JIT cache, no torch headers).

The shared library is the product boundary: a plain C ABI (include/b2p.h) over
hand-written CUDA. It is compiled from autoane_b200/csrc/*.cu, each object in
parallel, then linked with the static CUDA runtime.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libb2p.so"
OBJ_DIR = ROOT / "_build" / "obj"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"),
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the B200 library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max(f.stat().st_mtime for f in files)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link libb2p.so. Returns its path."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= _deps_mtime():
        build_host()
        return LIB
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr[-8000:]}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *map(str, objs),
           "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr[-8000:]}")
    os.replace(tmp, LIB)
    build_host()
    return LIB


HOST_SRC = PKG / "host" / "train_mezo.c"
HOST_EXE = PKG / "host" / "train_mezo"


def build_host(force: bool = False) -> Path:
    """The plain-C training loop (host/train_mezo.c) linked against libb2p.so."""
    if HOST_EXE.exists() and not force and HOST_EXE.stat().st_mtime >= max(
            HOST_SRC.stat().st_mtime, LIB.stat().st_mtime, (ROOT / "include" / "b2p.h").stat().st_mtime):
        return HOST_EXE
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler for the host loop")
    cmd = [cc, "-std=c11", "-O2", "-Wall", "-Wextra", "-I", str(ROOT / "include"), str(HOST_SRC), "-L", str(PKG),
           "-lb2p", "-Wl,-rpath,$ORIGIN/..", "-lm", "-o", str(HOST_EXE)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host loop build failed:\n{r.stderr[-4000:]}")
    return HOST_EXE


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
