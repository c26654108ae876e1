"""Pin the oracle (oracle/liboracle.so) to golden vectors produced by the
reference's own Python replicas (tests/golden/make_golden.py): the xoshiro256+
stream, Rademacher sign masks (4 bits per draw, 1-bit tails), the full-size
LoRA-layout masks, the fp32 perturbation chain and the cross-entropy."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

G = Path(__file__).resolve().parent / "golden"
PRNG = json.loads((G / "prng_golden.json").read_text())
CE = json.loads((G / "ce_golden.json").read_text())


@pytest.mark.parametrize("seed", list(PRNG["draws"].keys()))
def test_xoshiro_draws_match_reference_replica(seed):
    got = [format(v, "016x") for v in O.xo_draws(int(seed), 40)]
    assert got == PRNG["draws"][seed]


def test_ragged_buffers_tail_uses_one_draw_per_element():
    r = PRNG["ragged"]
    got = O.sign_mask(r["seed"], r["sizes"])
    assert [int(w) for w in got] == r["words"]


@pytest.mark.parametrize("name", list(PRNG["layouts"].keys()))
def test_lora_layout_masks(name):
    lay = PRNG["layouts"][name]
    L, D, Q, KV, r = lay["dims"][:5]
    H, ffn = lay["dims"][5:] if len(lay["dims"]) > 5 else (0, 0)
    sizes = O.lora_buffer_sizes_ffn(L, D, Q, KV, H, r, ffn)
    assert int(sizes.sum()) == lay["total"]
    for seed, ent in lay["masks"].items():
        m = O.sign_mask(int(seed), sizes)
        assert hashlib.sha256(m.astype("<u4").tobytes()).hexdigest() == ent["sha256"]
        assert [int(w) for w in m[:64]] == ent["head"]
        if "words" in ent:
            assert [int(w) for w in m] == ent["words"]


def test_smollm2_layout_size():
    lay = O.lora_layout(32, 960, 960, 320, 8)
    assert lay.layer_size == 53120 and lay.total == 1_700_800


def test_fp32_perturbation_chain_bit_exact():
    c = PRNG["chain"]
    buf = np.array(c["theta0"], dtype=np.uint32).view(np.float32).copy()
    eps, lr, g = np.float32(c["eps"]), np.float32(c["lr"]), np.float32(c["g"])
    for tag, scale in (("plus", eps), ("minus", np.float32(-2.0) * eps), ("restore", eps),
                       ("update", np.float32(-lr * g))):
        O.perturb_buffer(c["seed"], buf, scale)
        assert np.array_equal(buf.view(np.uint32), np.array(c[tag], dtype=np.uint32)), tag
    # the restore step is not an exact inverse in fp32 (reference behaviour)
    theta0 = np.array(c["theta0"], dtype=np.uint32).view(np.float32)
    restored = np.array(c["restore"], dtype=np.uint32).view(np.float32)
    assert np.abs(restored - theta0).max() < 1e-6


def test_perturb_lora_equals_mask_signs():
    L, D, Q, KV, r = 2, 64, 64, 32, 4
    sizes = O.lora_buffer_sizes(L, D, Q, KV, r)
    theta = np.zeros(int(sizes.sum()), np.float32)
    O.perturb_lora(theta, L, D, Q, KV, r, 99, 1.0)
    m = O.sign_mask(99, sizes)
    bits = (m[np.arange(theta.size) >> 5] >> (np.arange(theta.size) & 31).astype(np.uint32)) & 1
    assert np.array_equal(theta > 0, bits.astype(bool))


@pytest.mark.parametrize("case", range(len(CE["cases"])))
def test_cross_entropy_matches_reference_replica(case):
    c = CE["cases"][case]
    logits = np.array(c["logits"], np.uint32).view(np.float32).reshape(c["S"], c["V"])
    tg = np.array(c["targets"], np.uint16)
    lib = O.lib()
    import ctypes as C
    got = lib.or_cross_entropy(logits.ctypes.data_as(C.POINTER(C.c_float)),
                               tg.ctypes.data_as(C.POINTER(C.c_uint16)), c["V"], c["S"])
    assert abs(got - c["loss"]) <= 1e-6 * max(1.0, abs(c["loss"]))
