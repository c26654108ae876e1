"""The oracle's full-backprop gradient (or_full_grad, a restatement of train.m's
backward) against central finite differences of its own forward on a tiny model.
The P16 part of the same backward is pinned to the reference's compiled
bp_lora_backward in tests/test_oracle_vs_ref.py; this checks the added dW, RMS and
tied-embedding gradients. CPU only."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import _models as M

TINY = O.ModelCfg(dim=64, hidden=128, heads=2, kv_heads=1, hd=32, seq=16, nlayers=2, vocab=50, rank=4,
                  rope_theta=10000.0)


@pytest.fixture(scope="module")
def tiny():
    syn = M.make_model(TINY, n_active=40, seed=3, b_scale=0.0, rms_jitter=0.1, w_std=0.2)
    toks = M.make_tokens(2048, 40, seed=3)
    inp, tgt = M.sample_sequence(toks, TINY.seq, syn.full_to_compact, 11)
    return syn, inp, tgt


def loss_of(syn, weights, embed, theta, inp, tgt):
    cembed = np.ascontiguousarray(embed[syn.compact_to_full])
    om = O.OracleModel(TINY, weights, embed, cembed)
    return np.float64(om.forward_loss(theta, inp, tgt))


def fd(syn, inp, tgt, bump, h):
    wp, ep, tp = bump(+h)
    wm, em, tm = bump(-h)
    return (loss_of(syn, wp, ep, tp, inp, tgt) - loss_of(syn, wm, em, tm, inp, tgt)) / (2 * h)


def test_full_gradient_matches_finite_differences(tiny):
    syn, inp, tgt = tiny
    om = O.OracleModel(TINY, syn.weights, syn.embed, syn.cembed)
    loss, grad, dw, gembed = om.full_grad(syn.theta, inp, tgt, syn.compact_to_full)
    assert abs(loss - om.forward_loss(syn.theta, inp, tgt)) < 1e-6
    rng = np.random.default_rng(0)
    h = 1e-2
    for name in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"):
        for l in range(TINY.nlayers):
            d = rng.standard_normal(syn.weights[name][l].shape).astype(np.float32)
            d /= np.linalg.norm(d)

            def bump(s, name=name, l=l, d=d):
                w = {k: [a.copy() for a in v] for k, v in syn.weights.items()}
                w[name][l] = (w[name][l] + np.float32(s) * d).astype(np.float32)
                return w, syn.embed, syn.theta
            ref = fd(syn, inp, tgt, bump, h)
            got = float(np.sum(dw[name][l].astype(np.float64) * d))
            assert abs(got - ref) <= 2e-2 * max(abs(ref), 1e-2), (name, l, got, ref)
    # tied embedding: the input lookup and the compact classifier rows move together
    d = rng.standard_normal(syn.embed.shape).astype(np.float32)
    d /= np.linalg.norm(d)

    def bump_e(s):
        return syn.weights, (syn.embed + np.float32(s) * d).astype(np.float32), syn.theta
    ref = fd(syn, inp, tgt, bump_e, 2e-3)  # the embedding feeds a norm at 0.02 scale: more curvature
    got = float(np.sum(gembed.astype(np.float64) * d))
    assert abs(got - ref) <= 2e-2 * max(abs(ref), 1e-2), (got, ref)
    # RMS weights (theta layout)
    lay = syn.layout
    mask = np.zeros_like(syn.theta)
    for l in range(TINY.nlayers):
        b = l * lay.layer_size
        mask[b + lay.rms_att: b + lay.rms_ffn + TINY.dim] = 1
    mask[lay.rms_final: lay.rms_final + TINY.dim] = 1
    d = (rng.standard_normal(syn.theta.shape) * mask).astype(np.float32)
    d /= np.linalg.norm(d)

    def bump_t(s):
        return syn.weights, syn.embed, (syn.theta + np.float32(s) * d).astype(np.float32)
    ref = fd(syn, inp, tgt, bump_t, h)
    got = float(np.sum(grad.astype(np.float64) * d))
    assert abs(got - ref) <= 2e-2 * max(abs(ref), 1e-2), (got, ref)


def test_full_and_p16_share_the_lora_gradient(tiny):
    """With B = 0 the P16 adapter gradient equals the projection of the full dW (lora_grad_project)."""
    syn, inp, tgt = tiny
    om = O.OracleModel(TINY, syn.weights, syn.embed, syn.cembed)
    _, g16 = om.p16_grad(syn.theta, inp, tgt)
    _, gfull, dw, _ = om.full_grad(syn.theta, inp, tgt)
    assert np.array_equal(g16.view(np.uint32), gfull.view(np.uint32))
    lay, r = syn.layout, TINY.rank
    A = syn.theta[lay.Aq: lay.Aq + r * TINY.dim].reshape(r, TINY.dim)
    dBq = g16[lay.Bq: lay.Bq + TINY.q_dim * r].reshape(TINY.q_dim, r)
    assert np.allclose(dBq, dw["Wq"][0] @ A.T, rtol=1e-4, atol=1e-6)
