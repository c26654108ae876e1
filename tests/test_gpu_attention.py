"""Causal GQA attention on the tcgen05 kernel (csrc/attn_tc.cu) against the oracle
(causal SDPA of training/cpu_ops.h:321-360 through or_forward) and against the
mma.sync kernel it replaces, through the model's forward and backward, and the
tcgen05 attention backward (csrc/attn_bwd_tc.cu) against the mma.sync backward.

Tolerances: forward losses within 1e-3 nats of the oracle (fp16), 5e-3 (bf16);
the two device kernels within 2e-4 nats of each other (fp16; both round P to
16 bit, they differ in fp32 summation order). Backprop-LoRA gradients computed
from either kernel's saved row normalisers agree to 1e-2 relative L2, and so do
gradients from the two attention backward kernels (same loss, bit for bit: the
forward is the same).
Results do not depend on which CTA took which work unit: repeated launches are
bit-identical.
"""
import numpy as np
import pytest

from autoane_b200.model import BF16, F16, OPT_TC_ATTENTION, OPT_TC_ATTENTION_BWD
from tests import _models as M
from tests.test_gpu_model import make_pair, perturbed, seqs

pytestmark = pytest.mark.gpu

CASES = [
    ("smollm2_seq256_f16", M.small_cfg(nlayers=2, seq=256), F16, 1e-3),
    ("smollm2_seq256_bf16", M.small_cfg(nlayers=2, seq=256), BF16, 5e-3),
    ("autoresearch_seq128_f16", M.AUTORESEARCH, F16, 1e-3),
    ("smollm2_seq128_f16", M.small_cfg(nlayers=2, seq=128), F16, 1e-3),
]


@pytest.mark.parametrize("name,cfg,dtype,tol", CASES, ids=[c[0] for c in CASES])
def test_tc_attention_forward(b2p, name, cfg, dtype, tol):
    syn, om, model, toks = make_pair(cfg, dtype=dtype, max_groups=12)
    inp, tgt = seqs(syn, toks, 3, cfg.seq, base=500)
    seed, eps = 11, 1e-3
    variants = [(0, 0, 0.0, 0.0), (seed, 1, eps, 0.0), (seed, 2, eps, -2 * eps)]
    model.set_option(OPT_TC_ATTENTION, 1)
    got = model.eval(inp, tgt, variants)
    again = model.eval(inp, tgt, variants)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    model.set_option(OPT_TC_ATTENTION, 0)
    legacy = model.eval(inp, tgt, variants)
    model.set_option(OPT_TC_ATTENTION, 1)
    th_p = perturbed(syn.theta, cfg, seed, [eps])
    th_m = perturbed(syn.theta, cfg, seed, [eps, -2 * eps])
    ref = [np.mean([om.forward_loss(t, inp[i], tgt[i]) for i in range(3)]) for t in (syn.theta, th_p, th_m)]
    assert np.max(np.abs(got - ref)) < tol, (got, ref)
    if dtype == F16:
        assert np.max(np.abs(got - legacy)) < 2e-4, (got, legacy)
    model.close()


def test_tc_attention_p16_gradient_matches_legacy(b2p):
    cfg = M.small_cfg(nlayers=2, seq=256)
    syn, om, model, toks = make_pair(cfg, max_groups=4)
    inp, tgt = seqs(syn, toks, 2, cfg.seq, base=77)
    model.set_option(OPT_TC_ATTENTION, 1)
    l1, g1 = model.p16_grad(inp, tgt)
    model.set_option(OPT_TC_ATTENTION, 0)
    l0, g0 = model.p16_grad(inp, tgt)
    model.set_option(OPT_TC_ATTENTION, 1)
    assert abs(l1 - l0) < 2e-4
    rel = np.linalg.norm(g1.astype(np.float64) - g0) / np.linalg.norm(g0.astype(np.float64))
    assert rel < 1e-2, rel
    model.close()


@pytest.mark.parametrize("seq,dtype", [(256, F16), (128, F16), (256, BF16)])
def test_tc_attention_backward_matches_mma_sync(b2p, seq, dtype):
    cfg = M.small_cfg(nlayers=2, seq=seq)
    syn, om, model, toks = make_pair(cfg, dtype=dtype, max_groups=4)
    inp, tgt = seqs(syn, toks, 3, cfg.seq, base=91)
    model.set_option(OPT_TC_ATTENTION_BWD, 1)
    l1, g1 = model.p16_grad(inp, tgt)
    l1b, g1b = model.p16_grad(inp, tgt)
    model.set_option(OPT_TC_ATTENTION_BWD, 0)
    l0, g0 = model.p16_grad(inp, tgt)
    assert l1 == l0 and l1b == l1
    assert np.array_equal(g1.view(np.uint32), g1b.view(np.uint32))  # independent of the CTA work split
    rel = np.linalg.norm(g1.astype(np.float64) - g0) / np.linalg.norm(g0.astype(np.float64))
    assert rel < 1e-2, rel
    model.close()
