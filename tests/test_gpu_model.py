"""MeZO-LoRA-split path on the B200 against the oracle (oracle/oracle.c).

Tolerances (from the workload definition):
  * perturbation sign stream and fp32 update chain: bit-exact;
  * per-step loss: |L_gpu - L_oracle| < 1e-3 nats (fp16 compute), 5e-3 for bf16.
"""
import numpy as np
import pytest

from autoane_b200.model import BF16, F16, Config, Model, load_synthetic
from oracle import oracle as O
from tests import _models as M

pytestmark = pytest.mark.gpu

EPS = np.float32(1e-3)
LR = np.float32(1e-4)


def make_pair(cfg, dtype=F16, max_groups=16, n_active=3000, seed=7):
    syn = M.make_model(cfg, n_active=n_active, seed=seed, b_scale=0.01, rms_jitter=0.05)
    om = O.OracleModel(cfg, syn.weights, syn.embed, syn.cembed)
    mc = Config(dim=cfg.dim, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.hd,
                seq=cfg.seq, nlayers=cfg.nlayers, vocab=cfg.vocab, rank=cfg.rank, rope_theta=cfg.rope_theta,
                res_alpha=cfg.res_alpha, dtype=dtype, max_groups=max_groups)
    model = Model(mc)
    load_synthetic(model, syn.weights, syn.embed, syn.compact_to_full, syn.theta)
    toks = M.make_tokens(1 << 15, n_active, seed=seed)
    return syn, om, model, toks


def seqs(syn, toks, n, seq, base=100):
    inp, tgt = zip(*[M.sample_sequence(toks, seq, syn.full_to_compact, base + 977 * i) for i in range(n)])
    return np.stack(inp), np.stack(tgt)


@pytest.fixture(scope="module")
def small(b2p):
    cfg = M.small_cfg(nlayers=2, seq=128)
    return make_pair(cfg)


def perturbed(theta, cfg, seed, scales):
    t = theta.copy()
    for s in scales:
        O.perturb_lora(t, cfg.nlayers, cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.rank, seed, s)
    return t


def test_sign_masks_bit_exact_full_layout(b2p):
    model = Model(Config(max_groups=2))  # SmolLM2-360M layout, 1,700,800 trainable parameters
    assert model.P == 1_700_800
    seeds = [42, 1 * 1000003 + 42, 12345, 2**64 - 1, 7 * 1000003 + 42]
    got = model.sign_masks(seeds)
    sizes = O.lora_buffer_sizes(32, 960, 960, 320, 8)
    for i, s in enumerate(seeds):
        assert np.array_equal(got[i], O.sign_mask(s, sizes)), f"seed {s}"
    model.close()


def test_eval_unperturbed_matches_oracle(small):
    syn, om, model, toks = small
    cfg = syn.cfg
    inp, tgt = seqs(syn, toks, 3, cfg.seq)
    got = model.eval(inp, tgt, [(0, 0, 0.0, 0.0)])[0]
    ref = np.mean([om.forward_loss(syn.theta, inp[i], tgt[i]) for i in range(3)])
    assert abs(got - ref) < 1e-3, (got, ref)


def test_eval_perturbed_variants_match_oracle(small):
    syn, om, model, toks = small
    cfg = syn.cfg
    inp, tgt = seqs(syn, toks, 2, cfg.seq, base=5000)
    seed = 3 * 1000003 + 42
    vars_ = [(seed, 1, EPS, 0.0), (seed, 2, EPS, np.float32(-2.0) * EPS), (0, 0, 0.0, 0.0)]
    got = model.eval(inp, tgt, vars_)
    th_p = perturbed(syn.theta, cfg, seed, [EPS])
    th_m = perturbed(syn.theta, cfg, seed, [EPS, np.float32(-2.0) * EPS])
    ref = [np.mean([om.forward_loss(t, inp[i], tgt[i]) for i in range(2)]) for t in (th_p, th_m, syn.theta)]
    for g, r in zip(got, ref):
        assert abs(g - r) < 1e-3, (got, ref)


def test_mezo_step_update_chain_bit_exact(small):
    syn, om, model, toks = small
    cfg = syn.cfg
    model.set_trainable(syn.theta)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 777)
    seed = 9 * 1000003 + 42
    lp, lm, g = model.mezo_step(inp, tgt, seed, float(EPS), float(LR))
    th = syn.theta.copy()
    rlp, rlm, _ = om.mezo_step(th.copy(), inp, tgt, seed, float(EPS), float(LR))
    assert abs(lp - rlp) < 1e-3 and abs(lm - rlm) < 1e-3, (lp, lm, rlp, rlm)
    # the θ chain (+ε, -2ε, +ε, -lr·g) applied with the device's g must match bit for bit
    g32 = np.float32((np.float32(lp) - np.float32(lm)) / (np.float32(2.0) * EPS))
    assert np.float32(g) == g32
    ref_theta = perturbed(syn.theta, cfg, seed, [EPS, np.float32(-2.0) * EPS, EPS, np.float32(-LR * g32)])
    got_theta = model.get_trainable()
    assert np.array_equal(got_theta.view(np.uint32), ref_theta.view(np.uint32))
    model.set_trainable(syn.theta)


def test_dp_eval_and_update(small):
    syn, om, model, toks = small
    cfg = syn.cfg
    model.set_trainable(syn.theta)
    inp, tgt = seqs(syn, toks, 2, cfg.seq, base=9000)
    seeds = np.array([11 * 1000003 + 42, 11 * 1000003 + 43], np.uint64)
    pairs = model.mezo_eval(inp, tgt, seeds, float(EPS))
    for s_i, s in enumerate(seeds):
        for k, scales in enumerate(([EPS], [EPS, np.float32(-2.0) * EPS])):
            t = perturbed(syn.theta, cfg, int(s), scales)
            ref = np.mean([om.forward_loss(t, inp[i], tgt[i]) for i in range(2)])
            assert abs(pairs[2 * s_i + k] - ref) < 1e-3
    model.mezo_update(seeds, pairs, float(EPS), float(LR))
    ref_theta = syn.theta.copy()
    n = np.float32(len(seeds))
    for s_i, s in enumerate(seeds):
        g = np.float32((pairs[2 * s_i] - pairs[2 * s_i + 1]) / (np.float32(2.0) * EPS))
        c = np.float32(np.float32(-LR * g) / n)
        O.perturb_lora(ref_theta, cfg.nlayers, cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.rank, int(s), c)
    assert np.array_equal(model.get_trainable().view(np.uint32), ref_theta.view(np.uint32))
    model.set_trainable(syn.theta)


def test_bf16_eval_close(b2p):
    cfg = M.small_cfg(nlayers=2, seq=128)
    syn, om, model, toks = make_pair(cfg, dtype=BF16, max_groups=4)
    inp, tgt = seqs(syn, toks, 2, cfg.seq)
    got = model.eval(inp, tgt, [(0, 0, 0.0, 0.0)])[0]
    ref = np.mean([om.forward_loss(syn.theta, inp[i], tgt[i]) for i in range(2)])
    assert abs(got - ref) < 5e-3, (got, ref)
    model.close()


def test_full_smollm2_360m_step_matches_oracle(b2p):
    """SmolLM2-360M shapes (32 layers, SEQ 256, CV 16893): one MeZO step vs the oracle."""
    cfg = M.SMOLLM2
    syn, om, model, toks = make_pair(cfg, max_groups=2, n_active=16893, seed=42)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 12345)
    seed = 0 * 1000003 + 42
    lp, lm, g = model.mezo_step(inp, tgt, seed, float(EPS), float(LR))
    rlp, rlm, rg = om.mezo_step(syn.theta.copy(), inp, tgt, seed, float(EPS), float(LR))
    assert abs(lp - rlp) < 1e-3 and abs(lm - rlm) < 1e-3, (lp, lm, rlp, rlm)
    assert 9.0 < lp < 10.5  # ≈ ln(16893) for a random-init model (tests/test_training.sh step-0 band)
    model.close()


def test_pair_engine_seq256_matches_oracle_and_single_engine(b2p):
    """SEQ 256 puts every projection GEMM (with LoRA) on the CTA-pair engine."""
    cfg = M.small_cfg(nlayers=2, seq=256)
    syn, om, model, toks = make_pair(cfg, max_groups=8)
    inp, tgt = seqs(syn, toks, 2, cfg.seq, base=777)
    seed = 13 * 1000003 + 42
    vars_ = [(seed, 1, EPS, 0.0), (seed, 2, EPS, np.float32(-2.0) * EPS)]
    got_pair = model.eval(inp, tgt, vars_)
    from autoane_b200 import _lib
    _lib.call("b2p_model_set_option", model.h, 1, 0)
    got_single = model.eval(inp, tgt, vars_)
    _lib.call("b2p_model_set_option", model.h, 1, 1)
    th_p = perturbed(syn.theta, cfg, seed, [EPS])
    th_m = perturbed(syn.theta, cfg, seed, [EPS, np.float32(-2.0) * EPS])
    ref = [np.mean([om.forward_loss(t, inp[i], tgt[i]) for i in range(2)]) for t in (th_p, th_m)]
    for g, s, r in zip(got_pair, got_single, ref):
        assert abs(g - r) < 1e-3, (got_pair, ref)
        assert abs(g - s) < 2e-4, (got_pair, got_single)
    model.close()


def test_programmatic_dependent_launch_changes_no_result(b2p):
    """B2P_OPT_PDL only changes how kernels are launched: MeZO losses and the P16 gradient
    (forward, tcgen05 attention backward, elementwise backward kernels) are bit-identical
    with it on and off. The option is process-wide, so it is restored afterwards."""
    from autoane_b200.model import OPT_PDL
    cfg = M.small_cfg(nlayers=2, seq=256)
    syn, om, model, toks = make_pair(cfg, max_groups=8)
    inp, tgt = seqs(syn, toks, 2, cfg.seq, base=321)
    variants = [(0, 0, 0.0, 0.0), (5, 1, 1e-3, 0.0), (5, 2, 1e-3, -2e-3)]
    try:
        out = {}
        for pdl in (1, 0):
            model.set_option(OPT_PDL, pdl)
            out[pdl] = (model.eval(inp, tgt, variants), model.p16_grad(inp, tgt))
    finally:
        model.set_option(OPT_PDL, 1)
    assert np.array_equal(out[1][0].view(np.uint32), out[0][0].view(np.uint32))
    assert out[1][1][0] == out[0][1][0]
    assert np.array_equal(out[1][1][1].view(np.uint32), out[0][1][1].view(np.uint32))
    model.close()
