"""Checkpoint files on the host (no GPU work): the oracle restatement of BLZT v4 /
LORA reproduces the files pinned on the reference's reader (tests/golden/ckpt_golden.json,
made by tests/golden/make_ckpt_golden.py with generate.py's load_checkpoint), and the
library's header reader (b2p_ckpt_read_header, host only) accepts and rejects what the
reference's loaders do (train.m:211-229)."""
import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from autoane_b200 import _lib
from autoane_b200.model import read_checkpoint_header
from oracle import ckpt as K
from tests import _models as M

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "ckpt_golden.json").read_text())


def sha(p):
    return hashlib.sha256(Path(p).read_bytes()).hexdigest()


@pytest.fixture(scope="module")
def case():
    return M.ckpt_case(M.CKPT_TINY, GOLDEN["seed"])


def seeded_adam(layers, rms_final, embed, seed=11):
    rng = np.random.default_rng(seed)

    def mv(a):
        return (rng.standard_normal(np.shape(a)).astype(np.float32) * 1e-3,
                np.abs(rng.standard_normal(np.shape(a))).astype(np.float32) * 1e-6)
    return {"layers": [{k: mv(v) for k, v in lw.items()} for lw in layers], "rms_final": mv(rms_final),
            "embed": mv(embed)}


def test_oracle_writers_match_golden(case, tmp_path):
    layers, rms_final, embed, theta, lay = case
    cfg = M.CKPT_TINY
    hdr = GOLDEN["header"]
    p = tmp_path / "m.bin"
    K.write_blzt(p, dict(hdr, adam_t=0), layers, rms_final, embed)
    assert sha(p) == GOLDEN["blzt_mezo_sha256"] and p.stat().st_size == GOLDEN["blzt_mezo_bytes"]
    K.write_blzt(p, dict(hdr, adam_t=7), layers, rms_final, embed, seeded_adam(layers, rms_final, embed))
    assert sha(p) == GOLDEN["blzt_full_sha256"]
    back = K.read_blzt(p, cfg)
    assert back["header"]["adam_t"] == 7 and np.array_equal(back["embed"], embed)
    ad = K.adapters_of(theta, lay, cfg)
    K.write_lora(p, cfg.rank, 42, ad)
    assert sha(p) == GOLDEN["lora_sha256"]
    t, ad2 = K.read_lora(p, cfg)
    assert t == 42 and all(np.array_equal(a[k], b[k]) for a, b in zip(ad, ad2) for k in K.ADAPTERS)
    K.write_blzt(p, hdr, K.merged(layers, ad, +1.0), rms_final, embed)
    assert sha(p) == GOLDEN["blzt_merged_sha256"]


def test_header_struct_is_96_bytes():
    import ctypes as C
    assert C.sizeof(_lib.CkptHeader) == 96 == struct.calcsize(K.HDR_FMT)


def test_library_reads_header(case, tmp_path):
    layers, rms_final, embed, _, _ = case
    p = tmp_path / "m.bin"
    K.write_blzt(p, GOLDEN["header"], layers, rms_final, embed)
    got = read_checkpoint_header(p)
    assert got == GOLDEN["header"]


@pytest.mark.parametrize("field,value,status", [("magic", 0x46544B54, -1), ("version", 3, -1), ("step", -1, -1),
                                                ("step", 10000001, -1), ("adam_t", -5, -1)])
def test_library_rejects_bad_headers(tmp_path, field, value, status):
    p = tmp_path / "bad.bin"
    p.write_bytes(K.pack_header(dict(GOLDEN["header"], **{field: value})) + b"\0" * 64)
    with pytest.raises(_lib.B2PError) as e:
        read_checkpoint_header(p)
    assert e.value.rc == status


def test_library_rejects_truncated_and_missing(tmp_path):
    p = tmp_path / "short.bin"
    p.write_bytes(K.pack_header(GOLDEN["header"])[:50])
    with pytest.raises(_lib.B2PError) as e:
        read_checkpoint_header(p)
    assert e.value.rc == -6
    with pytest.raises(_lib.B2PError) as e:
        read_checkpoint_header(tmp_path / "absent.bin")
    assert e.value.rc == -6
