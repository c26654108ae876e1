"""The C ABI on the host (no GPU work): libb2p.so loads, exports every function
include/b2p.h declares, and the Python binding covers exactly that set."""
import ctypes as C
import re
from pathlib import Path

import pytest

from autoane_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b2p.h"


def declared():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(b2p_\w+)\s*\(", src))


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_matches_header():
    assert set(_lib.ABI) == declared()


def test_version_and_error_strings():
    lib = _lib.load()
    assert b"sm_100a" in lib.b2p_version()
    assert isinstance(lib.b2p_last_error(), bytes)


def test_struct_layouts_match_header():
    # b2p_model_config: 9 ints, 2 floats, 3 ints; b2p_variant: u64, int, 2 floats
    assert C.sizeof(_lib.ModelConfig) == 14 * 4
    assert C.sizeof(_lib.Variant) == 24


def test_missing_library_fails_loudly(tmp_path):
    saved = _lib._lib
    try:
        _lib._lib = None
        with pytest.raises(RuntimeError, match="no fallback"):
            _lib.load(tmp_path / "absent.so")
    finally:
        _lib._lib = saved


def test_io_shim_header_compiles_as_c(tmp_path):
    """include/b2p_io.h builds as C11 with warnings as errors (no GPU work)."""
    import subprocess
    for name in ("conv_fused_site.c", "dyn_site.c"):
        src = Path(__file__).resolve().parent / "shim" / name
        subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I", str(HEADER.parent),
                        str(src)], check=True)


def test_kern_compile_without_gpu_fails_loudly():
    """b2p_compile returns NULL with a reason when no B200 is usable; there is no CPU path."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from autoane_b200 import kern as KN
    import numpy as np
    with pytest.raises(_lib.B2PError):
        KN.compile_conv1x1_kern(np.zeros((64, 64), np.float32), 64, 64, 128)


def test_model_option_constants_match_header():
    """Every B2P_OPT_* macro of b2p.h has the same value as the binding's OPT_* constant."""
    from autoane_b200 import model
    opts = dict(re.findall(r"#define\s+B2P_OPT_(\w+)\s+(\d+)", HEADER.read_text()))
    assert {"PAIR_GEMM", "GRAD_SCALE_LOG2", "GRAPHS", "TC_ATTENTION", "TC_ATTENTION_BWD", "PDL"} <= set(opts)
    for name, value in opts.items():
        assert getattr(model, "OPT_" + name) == int(value), name
