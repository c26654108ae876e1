"""The plain-C host loop (autoane_b200/host/train_mezo.c) on the B200 against the same
steps driven from Python through the library.

The C program resumes from a BLZT file, builds the compact vocabulary from the
token file, draws the LoRA init and each step's position with the reference's
srand48/drand48 streams (training/train_mezo.m:1056-1093, 1946-1949) and runs
MeZO-LoRA-split (or backprop-LoRA) steps through libb2p. The Python side
restates the host work (oracle/sampling.py), calls the same library entry
points, and must reproduce every position, every loss and projected gradient
and the final trainable parameters bit for bit (the learning rates are taken
from the C program's trace; the restated schedule is checked to 1 ulp).
"""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from autoane_b200.model import Config, Model
from oracle import ckpt as CK
from oracle import oracle as O
from oracle import sampling as S

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
EXE = ROOT / "autoane_b200" / "host" / "train_mezo"
CFG = O.ModelCfg(dim=512, hidden=1408, heads=8, kv_heads=2, hd=64, seq=128, nlayers=2, vocab=49152, rank=8,
                 rope_theta=10000.0)  # training/models/autoresearch.h with 2 of its 4 layers


def f32_hex(s: str) -> np.float32:
    return np.float32(float.fromhex(s))


@pytest.fixture(scope="module")
def setup(b2p, tmp_path_factory):
    if not EXE.exists():
        pytest.fail(f"{EXE} is not built (autoane_b200/build.py builds it)")
    d = tmp_path_factory.mktemp("host")
    rng = np.random.default_rng(77)
    tokens = (rng.integers(0, 2000, 300_000) * 7 + 3).astype(np.uint16)  # sparse ids: a non-trivial compaction
    tokens.tofile(d / "tok.bin")
    D, H, QD, KVD = CFG.dim, CFG.hidden, CFG.q_dim, CFG.kv_dim
    shapes = {"Wq": (QD, D), "Wk": (KVD, D), "Wv": (KVD, D), "Wo": (D, QD), "W1": (H, D), "W2": (D, H), "W3": (H, D)}
    layers = []
    for _ in range(CFG.nlayers):
        lw = {k: (rng.standard_normal(s) * 0.02).astype(np.float32) for k, s in shapes.items()}
        lw["rms_att"] = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
        lw["rms_ffn"] = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
        layers.append(lw)
    rms_final = (1 + 0.05 * rng.standard_normal(D)).astype(np.float32)
    embed = (rng.standard_normal((CFG.vocab, D)) * 0.02).astype(np.float32)
    CK.write_blzt(d / "init.bin", CK.header(CFG, step=0, lr=3e-4, loss=0.0), layers, rms_final, embed)
    return d, tokens


def run_c(d, *extra):
    cmd = [str(EXE), "--model", "autoresearch", "--layers", "2", "--resume", str(d / "init.bin"), "--ckpt",
           str(d / "out.bin"), "--data", str(d / "tok.bin"), "--seed", "42", "--val-every", "0", "--trace",
           "--dump-theta", str(d / "theta.bin"), *extra]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    trace = []
    for line in r.stdout.splitlines():
        if line.startswith("trace "):
            trace.append(dict(kv.split("=", 1) for kv in line.split()[1:]))
    return trace, np.fromfile(d / "theta.bin", np.float32)


def python_model(d, tokens, max_groups):
    f2c, c2f = S.vocab_map_build(tokens, CFG.vocab)
    m = Model(Config(dim=CFG.dim, hidden=CFG.hidden, heads=CFG.heads, kv_heads=CFG.kv_heads, head_dim=CFG.hd,
                     seq=CFG.seq, nlayers=CFG.nlayers, vocab=CFG.vocab, rank=CFG.rank, rope_theta=CFG.rope_theta,
                     res_alpha=1.0, max_groups=max_groups))
    m.load_checkpoint(d / "init.bin", compact_to_full=c2f)
    theta = m.get_trainable()
    S.lora_init(theta, O.lora_layout(CFG.nlayers, CFG.dim, CFG.q_dim, CFG.kv_dim, CFG.rank), CFG, 42)
    m.set_trainable(theta)
    return m, f2c


def batch(tokens, f2c, pos):
    return tokens[pos:pos + CFG.seq].copy(), f2c[tokens[pos + 1:pos + 1 + CFG.seq]].astype(np.uint16)


def test_c_host_loop_mezo_matches_python_driven_steps(setup):
    d, tokens = setup
    trace, theta_c = run_c(d, "--lora-split", "--steps", "3", "--lr", "1e-4", "--epsilon", "1e-3")
    assert [int(t["step"]) for t in trace] == [0, 1, 2]
    m, f2c = python_model(d, tokens, 2)
    eps = float(np.float32(1e-3))
    for t in trace:
        s = int(t["step"])
        pos = S.train_position(42, s, len(tokens), CFG.seq)
        assert pos == int(t["pos"])
        assert int(t["seed"]) == s * 1000003 + 42
        lr = f32_hex(t["lr"])
        if s > 0:  # the schedule the C loop applied after step s-1, restated
            assert abs(int(S.mezo_lr(1e-4, s - 1, 0, 3).view(np.int32)) - int(lr.view(np.int32))) <= 1
        inp, tgt = batch(tokens, f2c, pos)
        lp, lm, g = m.mezo_step(inp, tgt, s * 1000003 + 42, eps, float(lr))
        assert np.float32(lp) == f32_hex(t["lp"]) and np.float32(lm) == f32_hex(t["lm"]), (s, lp, lm, t)
        assert np.float32(g) == f32_hex(t["g"])
    assert np.array_equal(m.get_trainable().view(np.uint32), theta_c.view(np.uint32))
    m.close()


def test_c_host_loop_backprop_lora_matches_python_driven_steps(setup):
    d, tokens = setup
    trace, theta_c = run_c(d, "--backprop-lora", "--steps", "2", "--lr", "3e-4")
    m, f2c = python_model(d, tokens, 1)
    m.set_adam_state(0, np.zeros(m.P, np.float32), np.zeros(m.P, np.float32))
    for t in trace:
        s = int(t["step"])
        pos = S.train_position(42, s, len(tokens), CFG.seq)
        assert pos == int(t["pos"])
        inp, tgt = batch(tokens, f2c, pos)
        loss = m.p16_step(inp[None], tgt[None], float(f32_hex(t["lr"])))
        assert np.float32(loss) == f32_hex(t["loss"]), (s, loss, t)
    assert np.array_equal(m.get_trainable().view(np.uint32), theta_c.view(np.uint32))
    m.close()
