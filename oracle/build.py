"""Build the oracle (CPU checker) libraries. TEST INFRASTRUCTURE ONLY.

  oracle/liboracle.so         our C restatement (oracle/oracle.c) + OpenBLAS
  oracle/_ref/libref_<m>.so   the reference's own training/cpu_ops.h and
                              training/backprop_lora.h compiled in place from the
                              AutoANE tree against oracle/shim (one per model header)
  oracle/_ref/validation_*    the reference's standalone C validators
                              (results/validation_*.c), compiled unchanged

The _ref part needs the reference tree, named by the AUTOANE_REF_ROOT
environment variable; without it (or where that tree is absent) the _ref part is
skipped, and prebuilt files already in oracle/_ref are used as they are.
Nothing here is used by libb2p.so.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_ROOT = Path(os.environ["AUTOANE_REF_ROOT"]) if os.environ.get("AUTOANE_REF_ROOT") else None
REF_OUT = HERE / "_ref"
LIBORACLE = HERE / "liboracle.so"
# reference model headers compiled into _ref (training/models/*.h) plus our own
# header for the 8/8-head, 1152-hidden variant of the 36.4M configuration
REF_MODELS = {
    "smollm2_360m": ("ref", "training/models/smollm2_360m.h"),
    "autoresearch": ("ref", "training/models/autoresearch.h"),
    "autoresearch_mha": ("here", "models/autoresearch_mha.h"),
}
CFLAGS = ["-O2", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-w"]


def find_openblas() -> Path:
    """Locate an LP64 OpenBLAS that exports cblas_sgemm (bundled inside a wheel on this image)."""
    env = os.environ.get("ORACLE_OPENBLAS")
    if env and Path(env).exists():
        return Path(env)
    import site
    roots = list(site.getsitepackages()) + [site.getusersitepackages()]
    for r in roots:
        for pat in ("*/libopenblas*.so*", "*.libs/libopenblas*.so*"):
            for cand in sorted(glob.glob(os.path.join(r, pat))):
                if "64_" in os.path.basename(cand):
                    continue  # ILP64 builds use suffixed symbol names
                return Path(cand)
    for cand in ("/usr/lib/x86_64-linux-gnu/libopenblas.so.0", "/usr/lib/libopenblas.so"):
        if os.path.exists(cand):
            return Path(cand)
    raise RuntimeError("no OpenBLAS with cblas_sgemm found for the oracle (set ORACLE_OPENBLAS)")


def _cc() -> str:
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("gcc not found")
    return cc


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{r.stderr[-4000:]}")


def _blas_link(blas: Path) -> list[str]:
    return [f"-L{blas.parent}", f"-l:{blas.name}", "-Wl,--disable-new-dtags", f"-Wl,-rpath,{blas.parent}", "-lm"]


def build_oracle(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if LIBORACLE.exists() and not force and LIBORACLE.stat().st_mtime >= max(
            src.stat().st_mtime, (HERE / "oracle.h").stat().st_mtime):
        return LIBORACLE
    blas = find_openblas()
    _run([_cc(), *CFLAGS, "-shared", str(src), "-o", str(LIBORACLE), *_blas_link(blas)])
    return LIBORACLE


def build_ref(force: bool = False) -> list[Path]:
    """Compile the reference's own C from REF_ROOT into oracle/_ref (skipped when absent)."""
    if REF_ROOT is None or not (REF_ROOT / "training" / "cpu_ops.h").exists():
        return []
    REF_OUT.mkdir(exist_ok=True)
    blas = find_openblas()
    out = []
    driver = HERE / "ref_driver.c"
    newest = max(p.stat().st_mtime for p in [driver, *(HERE / "shim").glob("*.h")])
    for name, (where, rel) in REF_MODELS.items():
        header = (REF_ROOT if where == "ref" else HERE) / rel
        lib = REF_OUT / f"libref_{name}.so"
        if lib.exists() and not force and lib.stat().st_mtime >= newest:
            out.append(lib)
            continue
        # -I<shim> -I- : quoted includes resolve in the shim first and never in the
        # including file's own directory, so the reference's Objective-C config.h /
        # io.h are replaced while cpu_ops.h / backprop_lora.h compile from REF_ROOT.
        _run([_cc(), *CFLAGS, "-shared", f"-I{HERE / 'shim'}", "-I-", f"-I{REF_ROOT / 'training'}",
              "-include", str(header), str(driver), "-o", str(lib), *_blas_link(blas)])
        out.append(lib)
    for v in ("validation_perturbation_cancel", "validation_gradient_unbiased"):
        exe = REF_OUT / v
        src = REF_ROOT / "results" / f"{v}.c"
        if src.exists() and (force or not exe.exists()):
            _run([_cc(), "-O2", "-w", str(src), "-o", str(exe), "-lm"])
        if exe.exists():
            out.append(exe)
    return out


def build(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIBORACLE, *sorted(p.name for p in REF_OUT.glob("*")) if REF_OUT.exists() else [])
