"""Full backprop (train.m) on the B200 against the oracle (or_full_grad, checked by
finite differences in tests/test_oracle_full.py).

The device trains fp32 masters made from its 16-bit weights, so the oracle is
given the same 16-bit-rounded weights. Tolerances as the P16 tests: per block
(each projection matrix of each layer, each RMS vector, the embedding) relative
L2 error < 5e-2 and cosine > 0.998; the AdamW update is bit-exact given the
device's own gradients when clipping does not engage.
"""
import numpy as np
import pytest

from autoane_b200.model import F16, Config, Model, load_synthetic
from oracle import oracle as O
from tests import _models as M
from tests.test_gpu_p16 import compare_grads

pytestmark = pytest.mark.gpu


def h16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def make_full(cfg, n_active=3000, seed=7, max_groups=4):
    syn = M.make_model(cfg, n_active=n_active, seed=seed, b_scale=0.0, rms_jitter=0.05)
    w16 = {k: [h16(a) for a in v] for k, v in syn.weights.items()}
    emb = syn.embed  # the lookup stays fp32 on the device; the classifier uses 16-bit rows
    om = O.OracleModel(cfg, w16, emb, h16(syn.cembed))
    mc = Config(dim=cfg.dim, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.hd,
                seq=cfg.seq, nlayers=cfg.nlayers, vocab=cfg.vocab, rank=cfg.rank, rope_theta=cfg.rope_theta,
                res_alpha=cfg.res_alpha, dtype=F16, max_groups=max_groups)
    model = Model(mc)
    load_synthetic(model, syn.weights, syn.embed, syn.compact_to_full, syn.theta)
    toks = M.make_tokens(1 << 15, n_active, seed=seed)
    return syn, om, model, toks


def block_check(name, got, ref, rel_tol=5e-2, cos_tol=0.998):
    g, r = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    rel = np.linalg.norm(g - r) / np.linalg.norm(r)
    cos = g @ r / (np.linalg.norm(g) * np.linalg.norm(r))
    assert rel < rel_tol and cos > cos_tol, f"{name}: rel {rel:.3e} cos {cos:.6f}"


@pytest.mark.parametrize("cfg", [M.AUTORESEARCH, M.small_cfg(nlayers=2, seq=256)], ids=["autoresearch", "smollm2x2"])
def test_full_gradients_match_oracle(b2p, cfg):
    syn, om, model, toks = make_full(cfg)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 41)
    loss = model.full_grad(inp[None], tgt[None])
    rloss, rgrad, rdw, rgemb = om.full_grad(syn.theta, inp, tgt, syn.compact_to_full)
    assert abs(loss - rloss) < 1e-3, (loss, rloss)
    dw = model.split_full_weights(model.full_read(Model.FULL_WEIGHT_GRADS))
    for name in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"):
        for l in range(cfg.nlayers):
            block_check(f"d{name}[{l}]", dw[name][l], rdw[name][l])
    block_check("dEmbed", model.full_read(Model.FULL_EMBED_GRAD).reshape(cfg.vocab, cfg.dim), rgemb)
    # RMS entries of the trainable-layout gradient
    g = model.full_read(Model.FULL_TRAINABLE_GRAD)
    lay = syn.layout
    for l in range(cfg.nlayers):
        b = l * lay.layer_size
        for off in (lay.rms_att, lay.rms_ffn):
            block_check(f"rms[{l}]", g[b + off: b + off + cfg.dim], rgrad[b + off: b + off + cfg.dim])
    block_check("rms_final", g[lay.rms_final: lay.rms_final + cfg.dim], rgrad[lay.rms_final: lay.rms_final + cfg.dim])
    # the masters start as the 16-bit weights
    w = model.split_full_weights(model.full_read(Model.FULL_WEIGHTS))
    assert np.array_equal(w["W2"][0], h16(syn.weights["W2"][0]))
    model.close()


def test_adamw_update_bit_exact_given_device_gradients(b2p):
    cfg = M.AUTORESEARCH
    syn, om, model, toks = make_full(cfg, seed=9)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 77)
    w0 = model.full_read(Model.FULL_WEIGHTS)
    e0 = model.full_read(Model.FULL_EMBED)
    model.full_grad(inp[None], tgt[None])
    gw = model.full_read(Model.FULL_WEIGHT_GRADS)
    ge = model.full_read(Model.FULL_EMBED_GRAD)
    gt = model.full_read(Model.FULL_TRAINABLE_GRAD)
    lr, wd = 3e-4, 0.1
    norm = model.full_update(lr, wd, clip=1e9)  # no clipping: the update is the plain AdamW step
    ref_norm = np.sqrt(np.sum(gw.astype(np.float64) ** 2) + np.sum(ge.astype(np.float64) ** 2) +
                       sum(np.sum(gt[sl].astype(np.float64) ** 2) for sl in M.rms_slices(syn)))
    assert abs(norm - ref_norm) <= 1e-4 * ref_norm
    w = w0.copy(); m = np.zeros_like(w); v = np.zeros_like(w)
    O.adam(w, gw, m, v, 1, lr, wd=wd)
    assert np.array_equal(model.full_read(Model.FULL_WEIGHTS).view(np.uint32), w.view(np.uint32))
    e = e0.copy(); m = np.zeros_like(e); v = np.zeros_like(e)
    O.adam(e, ge, m, v, 1, lr, wd=wd)
    assert np.array_equal(model.full_read(Model.FULL_EMBED).view(np.uint32), e.view(np.uint32))
    model.close()


def test_full_steps_reduce_loss_and_clip_bounds_norm(b2p):
    cfg = M.AUTORESEARCH
    syn, om, model, toks = make_full(cfg, seed=5)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 5)
    losses = []
    for _ in range(5):
        loss, norm = model.full_step(inp[None], tgt[None], 1e-3, wd=0.1, clip=1.0)
        losses.append(loss)
        assert np.isfinite(norm) and norm > 0
    assert losses[-1] < losses[0] - 1e-2, losses
    model.close()
