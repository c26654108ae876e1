"""Pin oracle/ckpt.py (the BLZT v4 / LORA restatement) on the reference's own reader.

Run once where the AutoANE reference tree is present, with AUTOANE_REF_ROOT
naming its root directory (required; the script refuses to guess a path):

    AUTOANE_REF_ROOT=<reference tree> python tests/golden/make_ckpt_golden.py

It writes a BLZT v4 file for the tiny case of tests/_models.py (CKPT_TINY,
ckpt_case seed 5) with oracle.ckpt.write_blzt, once with zero Adam slots (the
MeZO writer) and once with seeded Adam moments (the train.m writer), reads each
back with generate.py's load_checkpoint and checks every tensor, then records
the files' SHA-256 in ckpt_golden.json. It also records the SHA-256 of the
LORA sidecar of the same case. Tests read only the JSON.
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import io
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("AUTOANE_REF_ROOT"):
    sys.exit("set AUTOANE_REF_ROOT to the AutoANE reference tree")
REF = Path(os.environ["AUTOANE_REF_ROOT"])
sys.path.insert(0, str(ROOT))

from oracle import ckpt as K  # noqa: E402
from tests import _models as M  # noqa: E402


def _import(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    with contextlib.redirect_stdout(io.StringIO()):
        spec.loader.exec_module(mod)
    return mod


def seeded_adam(layers, rms_final, embed, seed=11):
    rng = np.random.default_rng(seed)

    def mv(a):
        return (rng.standard_normal(np.shape(a)).astype(np.float32) * 1e-3,
                np.abs(rng.standard_normal(np.shape(a))).astype(np.float32) * 1e-6)
    return {"layers": [{k: mv(v) for k, v in lw.items()} for lw in layers], "rms_final": mv(rms_final),
            "embed": mv(embed)}


def sha(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def main():
    gen = _import(REF / "generate.py", "ref_generate")
    cfg = M.CKPT_TINY
    layers, rms_final, embed, theta, lay = M.ckpt_case(cfg)
    hdr = K.header(cfg, step=123, total_steps=1000, lr=2.0 ** -12, loss=2.5, cum_train=10.5, cum_wall=20.25,
                   cum_steps=123)
    out = {"cfg": {k: getattr(cfg, k) for k in ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers",
                                                 "vocab", "rank")},
           "header": hdr, "seed": 5}
    with tempfile.TemporaryDirectory() as td:
        for name, adam in (("mezo", None), ("full", seeded_adam(layers, rms_final, embed))):
            p = Path(td) / f"{name}.bin"
            K.write_blzt(p, dict(hdr, adam_t=0 if adam is None else 7), layers, rms_final, embed, adam)
            conf, rl, rf, re = gen.load_checkpoint(str(p))
            assert conf["n_layers"] == cfg.nlayers and conf["dim"] == cfg.dim and conf["q_dim"] == cfg.q_dim
            for l in range(cfg.nlayers):
                for k, v in layers[l].items():
                    assert np.array_equal(rl[l][k], v), (name, l, k)
            assert np.array_equal(rf, rms_final) and np.array_equal(re, embed)
            back = K.read_blzt(p, cfg)
            assert back["header"] == dict(hdr, adam_t=0 if adam is None else 7)
            out[f"blzt_{name}_sha256"] = sha(p)
            out[f"blzt_{name}_bytes"] = p.stat().st_size
        lp = Path(td) / "lora.bin"
        K.write_lora(lp, cfg.rank, 42, K.adapters_of(theta, lay, cfg))
        t, ad = K.read_lora(lp, cfg)
        assert t == 42
        out["lora_sha256"] = sha(lp)
        mp = Path(td) / "merged.bin"
        K.write_blzt(mp, hdr, K.merged(layers, K.adapters_of(theta, lay, cfg), +1.0), rms_final, embed)
        out["blzt_merged_sha256"] = sha(mp)
    out["reader"] = "generate.py load_checkpoint"
    (HERE / "ckpt_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "ckpt_golden.json")


if __name__ == "__main__":
    main()
