"""The plain-C host loop (autoane_b200/host/train_mezo.c) on the host, no GPU work:
its data-sampling stream against the reference's formula (training/train_mezo.m:
1946-1949, restated in oracle/sampling.py), and that restatement's drand48 against
the libc drand48 the reference calls."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import sampling as S

ROOT = Path(__file__).resolve().parents[1]


def test_drand48_restatement_matches_libc():
    libc = C.CDLL(None)
    libc.drand48.restype = C.c_double
    libc.srand48.argtypes = [C.c_long]
    for seed in (42, 42 + 7919 * 3, 999, 42 + 12345, 2**33 + 5, 0):
        libc.srand48(seed)
        want = [libc.drand48() for _ in range(257)]
        g = S.Drand48(seed)
        got = [g.next() for _ in range(257)]
        assert got == want, seed
        g2 = S.Drand48(seed)
        assert np.array_equal(g2.fill(257), np.array(want))


def build_host(tmp_path) -> Path:
    exe = tmp_path / "train_mezo"
    subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "autoane_b200" / "host" / "train_mezo.c"), "-L", str(ROOT / "autoane_b200"),
                    "-lb2p", f"-Wl,-rpath,{ROOT / 'autoane_b200'}", "-lm", "-o", str(exe)], check=True)
    return exe


@pytest.mark.parametrize("n_tokens,model,seq", [(200_003, "autoresearch", 128), (1_000_000, "smollm2_360m", 256)])
def test_host_loop_positions_follow_reference_formula(tmp_path, n_tokens, model, seq):
    exe = build_host(tmp_path)
    tok = tmp_path / "tok.bin"
    np.random.default_rng(1).integers(0, 3000, n_tokens).astype(np.uint16).tofile(tok)
    for seed in (42, 7):
        out = subprocess.run([str(exe), "--model", model, "--data", str(tok), "--seed", str(seed), "--positions",
                              "64"], check=True, capture_output=True, text=True).stdout.split("\n")
        got = [int(line.split()[1]) for line in out if line.strip()]
        want = [S.train_position(seed, s, n_tokens, seq) for s in range(64)]
        assert got == want


def test_host_loop_rejects_unsupported_modes(tmp_path):
    exe = build_host(tmp_path)
    tok = tmp_path / "tok.bin"
    np.zeros(1000, np.uint16).tofile(tok)
    r = subprocess.run([str(exe), "--fzoo", "4", "--data", str(tok)], capture_output=True, text=True)
    assert r.returncode == 1 and "not part of this build" in r.stderr
    r = subprocess.run([str(exe), "--scratch", "--data", str(tok)], capture_output=True, text=True)
    assert r.returncode == 1 and "full-parameter MeZO" in r.stderr
    bad = tmp_path / "bad.bin"
    np.full(1000, 60000, np.uint16).tofile(bad)
    r = subprocess.run([str(exe), "--lora-split", "--scratch", "--data", str(bad)], capture_output=True, text=True)
    assert r.returncode == 1 and "VOCAB" in r.stderr
