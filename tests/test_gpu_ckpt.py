"""Checkpoints written and read by the device model, against the oracle's BLZT v4 /
LORA restatement (oracle/ckpt.py, pinned on the reference's generate.py reader).

  * a MeZO / P16 model writes byte-for-byte the file the oracle writes for the same
    tensors (frozen weights fp16-representable, so the widened 16-bit copies are exact);
  * with a sidecar, Wq/Wk/Wv/Wo are the merged W + B·A (fp32, k ascending) and the
    sidecar holds the adapters: byte-identical to the oracle;
  * loading restores weights, RMS vectors and embedding: the same losses bit for bit;
    loading with the sidecar un-merges (W - B·A, then the 16-bit upload);
  * a full-backprop model's file carries its masters and AdamW moments; a second model
    loaded from it continues training bit-identically.
"""
import numpy as np
import pytest

from autoane_b200 import _lib
from autoane_b200.model import F16, Config, Model, load_synthetic
from oracle import ckpt as K
from oracle import oracle as O
from tests import _models as M

pytestmark = pytest.mark.gpu

CFG = O.ModelCfg(dim=512, hidden=1408, heads=8, kv_heads=2, hd=64, seq=128, nlayers=2, vocab=4096, rank=8,
                 rope_theta=10000.0)
CV = 1000
HDR = dict(step=321, total_steps=5000, lr=2.0 ** -11, loss=3.25, cum_compile=1.5, cum_train=7.25, cum_wall=9.0,
           cum_steps=321, cum_batches=4)


def new_model(max_groups=4):
    return Model(Config(dim=CFG.dim, hidden=CFG.hidden, heads=CFG.heads, kv_heads=CFG.kv_heads, head_dim=CFG.hd,
                        seq=CFG.seq, nlayers=CFG.nlayers, vocab=CFG.vocab, rank=CFG.rank,
                        rope_theta=CFG.rope_theta, dtype=F16, max_groups=max_groups))


def weights_dict(layers):
    return {k: [lw[k] for lw in layers] for k in K.WEIGHTS}


@pytest.fixture(scope="module")
def case(b2p):
    layers, rms_final, embed, theta, lay = M.ckpt_case(CFG, seed=9)
    c2f = np.arange(CV, dtype=np.int32)
    model = new_model()
    load_synthetic(model, weights_dict(layers), embed, c2f, theta)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, CV, (2, CFG.seq + 1)).astype(np.uint16)
    yield layers, rms_final, embed, theta, lay, c2f, model, (toks[:, :-1].copy(), toks[:, 1:].copy())
    model.close()


def losses(model, batch):
    inp, tgt = batch
    return model.eval(inp, tgt, [(0, 0, 0.0, 0.0), (77, 1, 1e-3, 0.0)])


def test_mezo_save_is_the_reference_file(case, tmp_path):
    layers, rms_final, embed, theta, lay, c2f, model, _ = case
    p = tmp_path / "ckpt.bin"
    model.save_checkpoint(p, **HDR)
    q = tmp_path / "oracle.bin"
    K.write_blzt(q, K.header(CFG, **HDR), layers, rms_final, embed)
    assert p.read_bytes() == q.read_bytes()


def test_sidecar_and_merged_weights(case, tmp_path):
    layers, rms_final, embed, theta, lay, c2f, model, _ = case
    p, lp = tmp_path / "ckpt.bin", tmp_path / "ckpt_lora.bin"
    model.save_checkpoint(p, lora_path=lp, **HDR)
    ad = K.adapters_of(theta, lay, CFG)
    q, lq = tmp_path / "oracle.bin", tmp_path / "oracle_lora.bin"
    K.write_lora(lq, CFG.rank, 0, ad)
    K.write_blzt(q, K.header(CFG, **HDR), K.merged(layers, ad, +1.0), rms_final, embed)
    assert lp.read_bytes() == lq.read_bytes()
    assert p.read_bytes() == q.read_bytes()


def test_load_restores_the_model(case, tmp_path):
    layers, rms_final, embed, theta, lay, c2f, model, batch = case
    p = tmp_path / "ckpt.bin"
    model.save_checkpoint(p, **HDR)
    m2 = new_model()
    m2.set_trainable(np.where(np.arange(theta.size) % 3 == 0, 0.5, 0.0).astype(np.float32))
    # a model with no weights yet: the map comes with the call
    h = m2.load_checkpoint(p, compact_to_full=c2f)
    assert h["step"] == HDR["step"] and h["adam_t"] == 0 and h["q_dim"] == CFG.q_dim
    got = m2.get_trainable()
    D = CFG.dim
    for l in range(CFG.nlayers):
        s = slice(l * lay.layer_size + lay.rms_att, l * lay.layer_size + lay.rms_att + 2 * D)  # rms_att | rms_ffn
        assert np.array_equal(got[s], theta[s])
    assert np.array_equal(got[lay.rms_final:lay.rms_final + D], rms_final)
    m2.set_trainable(theta)
    assert np.array_equal(losses(m2, batch).view(np.uint32), losses(model, batch).view(np.uint32))
    m2.close()


def test_load_with_sidecar_unmerges(case, tmp_path):
    layers, rms_final, embed, theta, lay, c2f, model, batch = case
    p, lp = tmp_path / "ckpt.bin", tmp_path / "ckpt_lora.bin"
    model.save_checkpoint(p, lora_path=lp, **HDR)
    m2 = new_model()
    load_synthetic(m2, weights_dict(layers), embed, c2f, np.zeros_like(theta))
    m2.load_checkpoint(p, lora_path=lp)
    assert np.array_equal(m2.get_trainable().view(np.uint32), theta.view(np.uint32))
    t, _, _ = m2.adam_state()
    assert t == 0
    # the un-merged fp32 weights, rounded to 16 bit on upload, widened again on save
    ad = K.adapters_of(theta, lay, CFG)
    base = [{k: (v.astype(np.float16).astype(np.float32) if k in K.WEIGHTS else v) for k, v in lw.items()}
            for lw in K.merged(K.merged(layers, ad, +1.0), ad, -1.0)]
    r, q = tmp_path / "again.bin", tmp_path / "oracle.bin"
    m2.save_checkpoint(r, **HDR)
    K.write_blzt(q, K.header(CFG, **HDR), base, rms_final, embed)
    assert r.read_bytes() == q.read_bytes()
    m2.close()


def test_load_rejects_other_shapes(case, tmp_path):
    layers, rms_final, embed, theta, lay, c2f, model, _ = case
    p = tmp_path / "ckpt.bin"
    K.write_blzt(p, K.header(CFG, n_layers=3), layers + layers[:1], rms_final, embed)
    with pytest.raises(_lib.B2PError) as e:
        model.load_checkpoint(p)
    assert e.value.rc == -1
    K.write_blzt(p, K.header(CFG), layers, rms_final, embed)
    p.write_bytes(p.read_bytes()[:-4])  # one float short
    with pytest.raises(_lib.B2PError) as e:
        model.load_checkpoint(p)
    assert e.value.rc == -6


def test_full_mode_checkpoint_continues_training(b2p, tmp_path):
    layers, rms_final, embed, theta, lay = M.ckpt_case(CFG, seed=13)
    for l in range(CFG.nlayers):  # full backprop trains the weights; the adapters stay inert
        b = l * lay.layer_size
        for k, n in (("Bq", CFG.q_dim), ("Bk", CFG.kv_dim), ("Bv", CFG.kv_dim), ("Bo", CFG.dim)):
            theta[b + getattr(lay, k): b + getattr(lay, k) + n * CFG.rank] = 0
    c2f = np.arange(CV, dtype=np.int32)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, CV, (6, 2, CFG.seq + 1)).astype(np.uint16)
    m1 = new_model()
    load_synthetic(m1, weights_dict(layers), embed, c2f, theta)
    for i in range(2):
        m1.full_step(toks[i, :, :-1], toks[i, :, 1:], 1e-3)
    p = tmp_path / "full.bin"
    m1.save_checkpoint(p, **HDR)
    f = K.read_blzt(p, CFG)
    assert f["header"]["adam_t"] == 2
    w = m1.split_full_weights(m1.full_read(Model.FULL_WEIGHTS))
    for k in K.WEIGHTS:
        for l in range(CFG.nlayers):
            assert np.array_equal(f["layers"][l][k], w[k][l]), (k, l)
    assert np.array_equal(f["embed"].ravel(), m1.full_read(Model.FULL_EMBED))
    assert np.abs(f["adam"]["embed"][1]).max() > 0 and np.abs(f["adam"]["layers"][0]["W2"][0]).max() > 0

    m2 = new_model()
    load_synthetic(m2, weights_dict(layers), embed, c2f, theta)
    m2.load_checkpoint(p, full=True)
    for i in range(2, 4):
        l1, n1 = m1.full_step(toks[i, :, :-1], toks[i, :, 1:], 1e-3)
        l2, n2 = m2.full_step(toks[i, :, :-1], toks[i, :, 1:], 1e-3)
        assert l1 == l2 and n1 == n2, (i, l1, l2, n1, n2)
    assert np.array_equal(m1.full_read(Model.FULL_WEIGHTS).view(np.uint32),
                          m2.full_read(Model.FULL_WEIGHTS).view(np.uint32))
    assert np.array_equal(m1.get_trainable().view(np.uint32), m2.get_trainable().view(np.uint32))
    m1.close()
    m2.close()
