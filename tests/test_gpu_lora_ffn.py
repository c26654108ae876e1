"""--lora-ffn (LoRA adapters on W1, W2, W3 as well; train_mezo.m:866, 898) on the
B200 against the oracle (or_forward_loss with lora_ffn, pinned on the reference-code
forward in tests/test_oracle_vs_ref.py; sign stream pinned on the reference replica
in tests/test_oracle_golden.py).

  * sign masks over the FFN layout (4,404,160 parameters for SmolLM2-360M r8): bit-exact
  * losses of θ, θ+εz, θ-εz: within 1e-3 nats of the oracle (fp16)
  * the MeZO θ chain (+ε, -2ε, +ε, -lr·g): bit-exact
"""
import dataclasses

import numpy as np
import pytest

from autoane_b200 import _lib
from autoane_b200.model import F16, Config, Model, load_synthetic
from oracle import oracle as O
from tests import _models as M

pytestmark = pytest.mark.gpu

EPS = np.float32(1e-3)
LR = np.float32(1e-4)
CFG = dataclasses.replace(M.small_cfg(nlayers=2, seq=256), lora_ffn=True)


def perturbed(theta, cfg, seed, scales):
    t = theta.copy()
    for s in scales:
        O.perturb_lora_ffn(t, cfg.nlayers, cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.hidden, cfg.rank, True, seed, s)
    return t


def config(cfg, max_groups=8, **kw):
    return Config(dim=cfg.dim, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.hd,
                  seq=cfg.seq, nlayers=cfg.nlayers, vocab=cfg.vocab, rank=cfg.rank, rope_theta=cfg.rope_theta,
                  res_alpha=cfg.res_alpha, dtype=F16, max_groups=max_groups, lora_ffn=cfg.lora_ffn, **kw)


@pytest.fixture(scope="module")
def ffn(b2p):
    syn = M.make_model(CFG, n_active=3000, seed=11, b_scale=0.01, rms_jitter=0.05)
    om = O.OracleModel(CFG, syn.weights, syn.embed, syn.cembed)
    model = Model(config(CFG))
    load_synthetic(model, syn.weights, syn.embed, syn.compact_to_full, syn.theta)
    toks = M.make_tokens(1 << 15, 3000, seed=11)
    yield syn, om, model, toks
    model.close()


def seqs(syn, toks, n, seq, base):
    inp, tgt = zip(*[M.sample_sequence(toks, seq, syn.full_to_compact, base + 977 * i) for i in range(n)])
    return np.stack(inp), np.stack(tgt)


def test_sign_masks_ffn_layout_bit_exact(b2p):
    model = Model(Config(max_groups=2, lora_ffn=True))  # SmolLM2-360M with FFN adapters
    assert model.P == 4_404_160
    seeds = [42, 5 * 1000003 + 42, 2**64 - 1]
    got = model.sign_masks(seeds)
    sizes = O.lora_buffer_sizes_ffn(32, 960, 960, 320, 2560, 8, True)
    for i, s in enumerate(seeds):
        assert np.array_equal(got[i], O.sign_mask(s, sizes)), f"seed {s}"
    model.close()


def test_eval_variants_match_oracle(ffn):
    syn, om, model, toks = ffn
    inp, tgt = seqs(syn, toks, 2, CFG.seq, 300)
    seed = 7 * 1000003 + 42
    got = model.eval(inp, tgt, [(0, 0, 0.0, 0.0), (seed, 1, EPS, 0.0), (seed, 2, EPS, np.float32(-2.0) * EPS)])
    ths = (syn.theta, perturbed(syn.theta, CFG, seed, [EPS]),
           perturbed(syn.theta, CFG, seed, [EPS, np.float32(-2.0) * EPS]))
    ref = [np.mean([om.forward_loss(t, inp[i], tgt[i]) for i in range(2)]) for t in ths]
    assert np.max(np.abs(got - ref)) < 1e-3, (got, ref)
    # the FFN adapters matter: zeroing B1/B2/B3 changes the loss
    lay = syn.layout
    th0 = syn.theta.copy()
    for l in range(CFG.nlayers):
        b = l * lay.layer_size
        for off, n in ((lay.B1, CFG.hidden * CFG.rank), (lay.B2, CFG.dim * CFG.rank), (lay.B3, CFG.hidden * CFG.rank)):
            th0[b + off: b + off + n] = 0
    model.set_trainable(th0)
    l0 = model.eval(inp, tgt, [(0, 0, 0.0, 0.0)])[0]
    model.set_trainable(syn.theta)
    assert abs(l0 - got[0]) > 1e-4
    assert abs(l0 - np.mean([om.forward_loss(th0, inp[i], tgt[i]) for i in range(2)])) < 1e-3


def test_mezo_step_update_chain_bit_exact(ffn):
    syn, om, model, toks = ffn
    model.set_trainable(syn.theta)
    inp, tgt = M.sample_sequence(toks, CFG.seq, syn.full_to_compact, 4321)
    seed = 13 * 1000003 + 42
    lp, lm, g = model.mezo_step(inp, tgt, seed, float(EPS), float(LR))
    rlp, rlm, _ = om.mezo_step(syn.theta.copy(), inp, tgt, seed, float(EPS), float(LR))
    assert abs(lp - rlp) < 1e-3 and abs(lm - rlm) < 1e-3, (lp, lm, rlp, rlm)
    g32 = np.float32((np.float32(lp) - np.float32(lm)) / (np.float32(2.0) * EPS))
    assert np.float32(g) == g32
    ref_theta = perturbed(syn.theta, CFG, seed, [EPS, np.float32(-2.0) * EPS, EPS, np.float32(-LR * g32)])
    assert np.array_equal(model.get_trainable().view(np.uint32), ref_theta.view(np.uint32))
    model.set_trainable(syn.theta)


def test_unsupported_combinations_fail_loudly(ffn):
    syn, om, model, toks = ffn
    inp, tgt = M.sample_sequence(toks, CFG.seq, syn.full_to_compact, 5)
    with pytest.raises(_lib.B2PError):
        model.p16_grad(inp[None], tgt[None])
    with pytest.raises(_lib.B2PError):
        Model(config(dataclasses.replace(CFG, seq=128)))
