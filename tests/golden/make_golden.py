"""Generate the golden fixtures that pin the oracle (and through it the CUDA path).

Run once where the AutoANE reference tree is present, with AUTOANE_REF_ROOT
naming its root directory (required; the script refuses to guess a path):

    AUTOANE_REF_ROOT=<reference tree> python tests/golden/make_golden.py

It imports the reference's own Python replicas and writes small JSON files
next to this script; tests read only those JSON files:

  prng_golden.json  xoshiro256+/splitmix64 draws, Rademacher sign masks with 4-bit
                    draws and 1-bit tails, full-size LoRA-layout masks (digests) and
                    an fp32 perturbation chain (+eps, -2eps, +eps, -lr*g), all from
                    tools/verify_mezo_algorithm.py (Xoshiro256Plus, perturb_buffer_py)
  ce_golden.json    cross-entropy losses from tools/verify_ce_loss.py
                    (ce_loss_c_matching, the float32 replica of cpu_ops.h:108-133)
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import io
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
if not os.environ.get("AUTOANE_REF_ROOT"):
    sys.exit("set AUTOANE_REF_ROOT to the AutoANE reference tree")
REF = Path(os.environ["AUTOANE_REF_ROOT"])


def _import(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    with contextlib.redirect_stdout(io.StringIO()):
        spec.loader.exec_module(mod)  # verify_ce_loss.py runs its own checks at import
    return mod


def signs_to_words(signs: np.ndarray) -> list[int]:
    bits = (signs > 0).astype(np.uint8)
    n = len(bits)
    words = np.zeros((n + 31) // 32, dtype=np.uint64)
    idx = np.nonzero(bits)[0]
    np.bitwise_or.at(words, idx >> 5, (np.uint64(1) << (idx & 31).astype(np.uint64)))
    return [int(w) for w in words]


def lora_sizes(nlayers, dim, q_dim, kv_dim, r, hidden=0, ffn=False):
    """Buffer sizes in perturb_lora_weights order (train_mezo.m:566-587); the --lora-ffn
    adapters A1, B1, A2, B2, A3, B3 come after Bo."""
    sz = []
    for _ in range(nlayers):
        sz += [r * dim, q_dim * r, r * dim, kv_dim * r, r * dim, kv_dim * r, r * q_dim, dim * r]
        if ffn:
            sz += [r * dim, hidden * r, r * hidden, dim * r, r * dim, hidden * r]
        sz += [dim, dim]
    sz.append(dim)
    return sz


def mask_for(Xo, seed: int, sizes) -> list[int]:
    rng = Xo()
    rng.seed(seed)
    parts = [rng.rademacher_block(int(n)) for n in sizes]
    return signs_to_words(np.concatenate(parts))


def digest(words: list[int]) -> str:
    return hashlib.sha256(np.asarray(words, dtype="<u4").tobytes()).hexdigest()


def main() -> None:
    mz = _import(REF / "tools" / "verify_mezo_algorithm.py", "ref_verify_mezo")
    ce = _import(REF / "tools" / "verify_ce_loss.py", "ref_verify_ce")
    Xo = mz.Xoshiro256Plus

    out: dict = {"source": "tools/verify_mezo_algorithm.py (Xoshiro256Plus, perturb_buffer_py)"}
    # 1. raw draws
    draws = {}
    for seed in [0, 1, 42, 1000003 + 42, 42 * 1000003 + 42, 2**63 + 5, 2**64 - 1]:
        r = Xo()
        r.seed(seed)
        draws[str(seed)] = [format(r.next(), "016x") for _ in range(40)]
    out["draws"] = draws
    # 2. sign masks with ragged buffers (4-bit draws + 1-bit tails)
    ragged = [7, 13, 8, 1, 3, 4, 5, 0, 2]
    out["ragged"] = {"sizes": ragged, "seed": 12345, "words": mask_for(Xo, 12345, ragged)}
    # 3. full LoRA layouts
    layouts = {}
    for name, dims in {"smollm2_360m": (32, 960, 960, 320, 8),
                       "autoresearch": (4, 512, 512, 128, 8),
                       "autoresearch_r4": (4, 512, 512, 128, 4),
                       "smollm2_360m_lora_ffn": (32, 960, 960, 320, 8, 2560, 1)}.items():
        sizes = lora_sizes(*dims)
        seeds = [42, 1 * 1000003 + 42] if name == "smollm2_360m" else [42]
        layouts[name] = {"dims": list(dims), "total": int(sum(sizes)), "masks": {}}
        for s in seeds:
            w = mask_for(Xo, s, sizes)
            entry = {"sha256": digest(w), "head": w[:64], "tail": w[-16:]}
            if not name.startswith("smollm2_360m"):
                entry["words"] = w
            layouts[name]["masks"][str(s)] = entry
    out["layouts"] = layouts
    # 4. fp32 perturbation chain on a small buffer, as the MeZO step applies it
    rng = np.random.default_rng(7)
    theta0 = (rng.standard_normal(66) * 0.3).astype(np.float32)
    eps, lr, g = np.float32(1e-3), np.float32(1e-4), np.float32(5.407333)
    seed = 5 * 1000003 + 42
    buf = theta0.copy()
    chain = {"theta0": [int(v) for v in theta0.view(np.uint32)]}
    for tag, scale in (("plus", eps), ("minus", np.float32(-2.0) * eps), ("restore", eps),
                       ("update", np.float32(-lr * g))):
        r = Xo()
        r.seed(seed)
        z = r.rademacher_block(len(buf))
        buf = (buf.astype(np.float64) + np.float64(scale) * z).astype(np.float32)
        chain[tag] = [int(v) for v in buf.view(np.uint32)]
    chain.update({"seed": seed, "eps": float(eps), "lr": float(lr), "g": float(g)})
    out["chain"] = chain
    (HERE / "prng_golden.json").write_text(json.dumps(out))

    # CE golden
    rng = np.random.default_rng(11)
    cases = []
    for S, V in [(4, 10), (8, 257), (16, 1000)]:
        logits = (rng.standard_normal((S, V)) * 3).astype(np.float32)
        tg = rng.integers(0, V, S).astype(np.uint16)
        loss, _ = ce.ce_loss_c_matching(logits, tg)
        cases.append({"S": S, "V": V, "logits": [int(v) for v in logits.view(np.uint32).ravel()],
                      "targets": tg.tolist(), "loss": float(loss)})
    (HERE / "ce_golden.json").write_text(json.dumps({"source": "tools/verify_ce_loss.py ce_loss_c_matching",
                                                     "cases": cases}))
    print("wrote", HERE / "prng_golden.json", HERE / "ce_golden.json")


if __name__ == "__main__":
    sys.exit(main())
