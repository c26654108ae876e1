"""Pin the oracle restatement to the reference's own C, compiled in place from
the AutoANE tree (oracle/_ref, built by oracle/build.py): cpu_ops.h's rmsnorm,
rope, SDPA and cross-entropy, and the DO_FORWARD_PASS transcription over them.
Skipped where oracle/_ref was not built (no reference tree at build time)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests import _models as M

F = C.POINTER(C.c_float)


def f(a):
    return a.ctypes.data_as(F)


def need(model):
    lib = O.ref_lib(model)
    if lib is None:
        pytest.skip("oracle/_ref not built (reference tree absent at build time)")
    return lib


def test_rmsnorm_rope_sdpa_ce_bit_exact():
    ref = need("autoresearch")
    rng = np.random.default_rng(3)
    d, S, hd, heads = 512, 128, 64, 8
    x = rng.standard_normal((d, S), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    a, b = np.zeros_like(x), np.zeros_like(x)
    ref.ref_rmsnorm(f(a), f(x), f(w), d, S)
    O.lib().or_rmsnorm(f(b), f(x), f(w), d, S)
    assert np.array_equal(a, b)
    q1, q2 = x.copy(), x.copy()
    ref.ref_rope_forward(f(q1), S, d, hd)  # autoresearch header: default ROPE_THETA 10000
    O.lib().or_rope_forward(f(q2), S, d, hd, C.c_float(10000.0))
    assert np.array_equal(q1, q2)
    K = rng.standard_normal((d, S), dtype=np.float32)
    V = rng.standard_normal((d, S), dtype=np.float32)
    o1, o2 = np.zeros_like(x), np.zeros_like(x)
    ref.ref_sdpa_forward(f(x), f(K), f(V), f(o1), heads, hd, S)
    O.lib().or_sdpa_forward(f(x), f(K), f(V), f(o2), heads, hd, S)
    assert np.array_equal(o1, o2)
    logits = (3 * rng.standard_normal((S, 777))).astype(np.float32)
    tg = rng.integers(0, 777, S).astype(np.uint16)
    dl = np.zeros_like(logits)
    u16 = tg.ctypes.data_as(C.POINTER(C.c_uint16))
    l1 = ref.ref_cross_entropy(f(dl), f(logits), u16, 777, S)
    l2 = O.lib().or_cross_entropy(f(logits), u16, 777, S)
    assert l1 == l2


@pytest.mark.parametrize("model,cfg", [("autoresearch", M.AUTORESEARCH), ("autoresearch_mha", M.AUTORESEARCH_MHA)])
def test_forward_loss_matches_reference_code(model, cfg):
    ref = need(model)
    syn = M.make_model(cfg, n_active=3000, seed=5, b_scale=0.01, rms_jitter=0.05)
    toks = M.make_tokens(4096, 3000, seed=5)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 17)
    om = O.OracleModel(cfg, syn.weights, syn.embed, syn.cembed)
    loss_o = om.forward_loss(syn.theta, inp, tgt)
    L, lay = cfg.nlayers, syn.layout
    keep = []

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p

    lora, rms = [], []
    for l in range(L):
        base = l * lay.layer_size
        for off in (lay.Aq, lay.Bq, lay.Ak, lay.Bk, lay.Av, lay.Bv, lay.Ao, lay.Bo):
            lora.append(syn.theta[base + off:])
        rms += [syn.theta[base + lay.rms_att:], syn.theta[base + lay.rms_ffn:]]
    lora = [np.ascontiguousarray(a) for a in lora]
    rms = [np.ascontiguousarray(a) for a in rms]
    ref.ref_forward_loss.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                          C.POINTER(C.c_uint16), C.POINTER(C.c_uint16)]
    rf = np.ascontiguousarray(syn.theta[lay.rms_final:])
    loss_r = ref.ref_forward_loss(*[plist(syn.weights[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")],
                                  plist(lora), plist(rms), f(rf), f(syn.embed), f(syn.cembed), syn.cembed.shape[0],
                                  cfg.rank, C.c_float(cfg.res_alpha), inp.ctypes.data_as(C.POINTER(C.c_uint16)),
                                  tgt.ctypes.data_as(C.POINTER(C.c_uint16)))
    assert abs(loss_o - loss_r) < 1e-5, (loss_o, loss_r)
    assert 7.0 < loss_o < 9.0  # ≈ ln(3000) for a random-init model


def test_forward_loss_lora_ffn_matches_reference_code():
    """--lora-ffn forward (adapters on W1, W2, W3) against the reference code path."""
    import dataclasses
    ref = need("autoresearch")
    cfg = dataclasses.replace(M.AUTORESEARCH, lora_ffn=True)
    syn = M.make_model(cfg, n_active=3000, seed=6, b_scale=0.01, rms_jitter=0.05)
    toks = M.make_tokens(4096, 3000, seed=6)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 23)
    om = O.OracleModel(cfg, syn.weights, syn.embed, syn.cembed)
    loss_o = om.forward_loss(syn.theta, inp, tgt)
    plain = dataclasses.replace(cfg, lora_ffn=False)
    keep = []

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p

    lay = syn.layout
    lora, rms, ffn = [], [], []
    for l in range(cfg.nlayers):
        base = l * lay.layer_size
        lora += [np.ascontiguousarray(syn.theta[base + o:]) for o in (lay.Aq, lay.Bq, lay.Ak, lay.Bk, lay.Av, lay.Bv,
                                                                       lay.Ao, lay.Bo)]
        ffn += [np.ascontiguousarray(syn.theta[base + o:]) for o in (lay.A1, lay.B1, lay.A2, lay.B2, lay.A3, lay.B3)]
        rms += [np.ascontiguousarray(syn.theta[base + o:]) for o in (lay.rms_att, lay.rms_ffn)]
    ref.ref_forward_loss_ffn.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                              C.POINTER(C.c_uint16), C.POINTER(C.c_uint16),
                                                              C.POINTER(F)]
    rf = np.ascontiguousarray(syn.theta[lay.rms_final:])
    loss_r = ref.ref_forward_loss_ffn(*[plist(syn.weights[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")],
                                      plist(lora), plist(rms), f(rf), f(syn.embed), f(syn.cembed),
                                      syn.cembed.shape[0], cfg.rank, C.c_float(cfg.res_alpha),
                                      inp.ctypes.data_as(C.POINTER(C.c_uint16)),
                                      tgt.ctypes.data_as(C.POINTER(C.c_uint16)), plist(ffn))
    assert abs(loss_o - loss_r) < 1e-5, (loss_o, loss_r)
    # the FFN adapters change the loss (they are not inert)
    th0 = np.zeros(O.lora_layout(plain.nlayers, plain.dim, plain.q_dim, plain.kv_dim, plain.rank).total, np.float32)
    lay0 = O.lora_layout(plain.nlayers, plain.dim, plain.q_dim, plain.kv_dim, plain.rank)
    for l in range(cfg.nlayers):
        b0, b = l * lay0.layer_size, l * lay.layer_size
        th0[b0: b0 + lay0.rms_att] = syn.theta[b: b + lay.Bo + cfg.dim * cfg.rank]
        th0[b0 + lay0.rms_att: b0 + lay0.layer_size] = syn.theta[b + lay.rms_att: b + lay.layer_size]
    th0[lay0.rms_final:] = syn.theta[lay.rms_final:]
    loss_plain = O.OracleModel(plain, syn.weights, syn.embed, syn.cembed).forward_loss(th0, inp, tgt)
    assert abs(loss_plain - loss_o) > 1e-5


def _theta_lists(syn, L):
    lay = syn.layout
    lora, rms = [], []
    for l in range(L):
        base = l * lay.layer_size
        for off in (lay.Aq, lay.Bq, lay.Ak, lay.Bk, lay.Av, lay.Bv, lay.Ao, lay.Bo):
            lora.append(syn.theta[base + off:])
        rms += [syn.theta[base + lay.rms_att:], syn.theta[base + lay.rms_ffn:]]
    return [np.ascontiguousarray(a) for a in lora], [np.ascontiguousarray(a) for a in rms]


@pytest.mark.parametrize("model,cfg", [("autoresearch", M.AUTORESEARCH), ("autoresearch_mha", M.AUTORESEARCH_MHA)])
def test_p16_gradient_matches_reference_backward(model, cfg):
    """or_p16_grad against the reference's bp_lora_backward (backprop_lora.h:147-288) compiled in place."""
    ref = need(model)
    syn = M.make_model(cfg, n_active=3000, seed=11, b_scale=0.02, rms_jitter=0.05)
    toks = M.make_tokens(4096, 3000, seed=11)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 23)
    om = O.OracleModel(cfg, syn.weights, syn.embed, syn.cembed)
    loss_o, grad_o = om.p16_grad(syn.theta, inp, tgt)
    L, lay, r, D = cfg.nlayers, syn.layout, cfg.rank, cfg.dim
    keep = []

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p

    lora, rms = _theta_lists(syn, L)
    sizes = [r * D, cfg.q_dim * r, r * D, cfg.kv_dim * r, r * D, cfg.kv_dim * r, r * cfg.q_dim, D * r]
    glora = [np.zeros(sizes[k % 8], np.float32) for k in range(8 * L)]
    grms = [np.zeros(D, np.float32) for _ in range(2 * L)]
    grf = np.zeros(D, np.float32)
    rf = np.ascontiguousarray(syn.theta[lay.rms_final:])
    ref.ref_p16_grad.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                      C.POINTER(C.c_uint16), C.POINTER(C.c_uint16),
                                                      C.POINTER(F), C.POINTER(F), F]
    loss_r = ref.ref_p16_grad(*[plist(syn.weights[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")],
                              plist(lora), plist(rms), f(rf), f(syn.embed), f(syn.cembed), syn.cembed.shape[0], r,
                              C.c_float(cfg.res_alpha), inp.ctypes.data_as(C.POINTER(C.c_uint16)),
                              tgt.ctypes.data_as(C.POINTER(C.c_uint16)), plist(glora), plist(grms), f(grf))
    assert abs(loss_o - loss_r) < 1e-5, (loss_o, loss_r)
    grad_r = np.zeros_like(grad_o)
    offs = (lay.Aq, lay.Bq, lay.Ak, lay.Bk, lay.Av, lay.Bv, lay.Ao, lay.Bo)
    for l in range(L):
        base = l * lay.layer_size
        for k, off in enumerate(offs):
            grad_r[base + off: base + off + sizes[k]] = glora[8 * l + k]
        grad_r[base + lay.rms_att: base + lay.rms_att + D] = grms[2 * l]
        grad_r[base + lay.rms_ffn: base + lay.rms_ffn + D] = grms[2 * l + 1]
    grad_r[lay.rms_final: lay.rms_final + D] = grf
    # same fp32 arithmetic through the same BLAS; only summation order differs
    err = np.abs(grad_o - grad_r).max()
    assert err <= 1e-4 * np.abs(grad_r).max(), (err, np.abs(grad_r).max())
    assert np.abs(grad_r).max() > 0


def test_adam_matches_reference_bit_exact():
    ref = need("autoresearch")
    rng = np.random.default_rng(4)
    n = 10007
    w0 = rng.standard_normal(n).astype(np.float32)
    m0 = (0.01 * rng.standard_normal(n)).astype(np.float32)
    v0 = (0.001 * rng.random(n)).astype(np.float32)
    for t in (1, 2, 37):
        g = (0.1 * rng.standard_normal(n)).astype(np.float32)
        w1, m1, v1 = w0.copy(), m0.copy(), v0.copy()
        w2, m2, v2 = w0.copy(), m0.copy(), v0.copy()
        ref.ref_adam(f(w1), f(g), f(m1), f(v1), C.c_size_t(n), t, C.c_float(3e-4), C.c_float(0.9),
                     C.c_float(0.95), C.c_float(1e-8), C.c_float(0.0))
        O.adam(w2, g, m2, v2, t, 3e-4)
        assert np.array_equal(w1.view(np.uint32), w2.view(np.uint32))
        assert np.array_equal(m1.view(np.uint32), m2.view(np.uint32))
        assert np.array_equal(v1.view(np.uint32), v2.view(np.uint32))


@pytest.mark.parametrize("model,cfg", [("autoresearch", M.AUTORESEARCH), ("autoresearch_mha", M.AUTORESEARCH_MHA)])
def test_full_grad_dw_matches_reference_materialised_dw(model, cfg):
    """Config 0 (full backprop, train.m) weight gradients of Wq/Wk/Wv/Wo against the dW
    matrices the reference's compiled bp_lora_backward materialises before projecting them
    onto the adapters (training/backprop_lora.h:223-270). With B = 0 the merged weights are
    the base weights, so both are dL/dW of the same network. res_alpha 1/sqrt(2L) as the
    from-scratch configuration scales its residual branches (train.m DeepNet init)."""
    import dataclasses
    ref = need(model)
    cfg = dataclasses.replace(cfg, res_alpha=float(np.float32(1.0 / np.sqrt(2 * cfg.nlayers))))
    syn = M.make_model(cfg, n_active=3000, seed=13, b_scale=0.0, rms_jitter=0.05, w_std=0.05)
    toks = M.make_tokens(4096, 3000, seed=13)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 41)
    om = O.OracleModel(cfg, syn.weights, syn.embed, syn.cembed)
    loss_o, _, dw_o, _ = om.full_grad(syn.theta, inp, tgt)
    L, lay, r, D, QD, KVD = cfg.nlayers, syn.layout, cfg.rank, cfg.dim, cfg.q_dim, cfg.kv_dim
    keep = []

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p

    lora, rms = _theta_lists(syn, L)
    sizes = [r * D, QD * r, r * D, KVD * r, r * D, KVD * r, r * QD, D * r]
    glora = [np.zeros(sizes[k % 8], np.float32) for k in range(8 * L)]
    grms = [np.zeros(D, np.float32) for _ in range(2 * L)]
    grf = np.zeros(D, np.float32)
    rf = np.ascontiguousarray(syn.theta[lay.rms_final:])
    per_layer = [("Wo", (D, QD)), ("Wq", (QD, D)), ("Wk", (KVD, D)), ("Wv", (KVD, D))]
    dw = np.zeros(L * sum(a * b for _, (a, b) in per_layer), np.float32)
    ref.ref_p16_grad_dw.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                         C.POINTER(C.c_uint16), C.POINTER(C.c_uint16),
                                                         C.POINTER(F), C.POINTER(F), F, F]
    loss_r = ref.ref_p16_grad_dw(*[plist(syn.weights[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")],
                                 plist(lora), plist(rms), f(rf), f(syn.embed), f(syn.cembed), syn.cembed.shape[0], r,
                                 C.c_float(cfg.res_alpha), inp.ctypes.data_as(C.POINTER(C.c_uint16)),
                                 tgt.ctypes.data_as(C.POINTER(C.c_uint16)), plist(glora), plist(grms), f(grf), f(dw))
    assert abs(loss_o - loss_r) < 1e-5, (loss_o, loss_r)
    o, worst = 0, 0.0
    for l in reversed(range(L)):
        for name, (a, b) in per_layer:
            got, want = dw_o[name][l].astype(np.float64), dw[o:o + a * b].reshape(a, b)
            o += a * b
            assert np.linalg.norm(want) > 0, (name, l)
            e = np.linalg.norm(got - want) / np.linalg.norm(want)
            worst = max(worst, e)
            # same fp32 arithmetic through the same BLAS; only summation order differs
            assert e < 1e-4, (name, l, e)
    assert o == dw.size
