"""Projection outputs against the reference CPU path on identical fp32 inputs.

The reference's CPU path multiplies fp32 weights and activations with
cblas_sgemm (training/train_mezo.m:1533-1538, 1598, 1630-1692) and adds the
adapters with lora_addmm (:694-703). Here the oracle gets exactly those fp32
inputs, unrounded; the device rounds them to fp16 at the boundary (as the
reference's Neural-Engine path does on write, training/io.h:42-51) and
accumulates in fp32. The gate is the workload's projection tolerance:

    max |y_dev - y_ref| / max |y_ref|  <  2e-3        (fp16 compute)

measured over the whole output of each operator. For fp16 inputs of unit
roundoff 2^-11 the expected value is about 1e-4 per GEMM: every product w·x
carries a relative error below 2^-10, the errors of a K-term sum add like a
random walk, and the largest output element is several standard deviations
of the sum. The FFN chains three GEMMs through a 16-bit gate, the qkv case
adds the 16-bit LoRA-down result and the LoRA-up product.
"""
import numpy as np
import pytest

from autoane_b200 import kern as KN
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3


def rnd(rng, shape, std=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)


def max_rel(got, ref):
    return float(np.max(np.abs(got.astype(np.float64) - ref)) / np.max(np.abs(ref)))


SHAPES = [("Wq/Wo", 960, 960), ("Wk/Wv", 320, 960), ("W1/W3", 2560, 960), ("W2", 960, 2560)]


@pytest.mark.parametrize("S", [128, 256, 1024])
@pytest.mark.parametrize("name,oc,ic", SHAPES, ids=[s[0] for s in SHAPES])
def test_projection_fp32_inputs(b2p, name, oc, ic, S):
    rng = np.random.default_rng(oc * 7 + ic + S)
    W, x = rnd(rng, (oc, ic), 0.02), rnd(rng, (ic, S))  # workload values: N(0, 0.02^2) weights, N(0, 1) activations
    k = KN.compile_conv1x1_kern(W, ic, oc, S)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    e = max_rel(KN.io_read_dyn(k), O.sgemm(W, x))
    KN.free_kern(k)
    print(f"{name} S={S}: max rel err {e:.2e}")
    assert e < TOL, e


def test_qkv_lora_fp32_inputs(b2p):
    rng = np.random.default_rng(17)
    D, Q, KV, S, r = 960, 960, 320, 256, 8
    Ws = [rnd(rng, (o, D), 0.02) for o in (Q, KV, KV)]
    x = rnd(rng, (D, S))
    params = [(rnd(rng, (r, D), 1.0 / np.sqrt(r)), rnd(rng, (o, r), 0.01)) for o in (Q, KV, KV)]
    k = KN.compile_qkv_fused_conv1x1_kern(*Ws, D, Q, KV, S)
    for i, (A, B) in enumerate(params):
        k.set_lora(i, A, B, r)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    row, worst = 0, 0.0
    for W, (A, B), o in zip(Ws, params, (Q, KV, KV)):
        ref = O.sgemm(W, x)
        O.lora_addmm(ref, A, B, x)  # train_mezo.m:1541-1543
        worst = max(worst, max_rel(y[row:row + o], ref))
        row += o
    k.free()
    print(f"qkv + LoRA: max rel err {worst:.2e}")
    assert worst < TOL, worst


@pytest.mark.parametrize("S", [128, 256])
def test_ffn_fp32_inputs(b2p, S):
    rng = np.random.default_rng(S + 1)
    D, H = 960, 2560
    W1, W3, W2 = rnd(rng, (H, D), 0.02), rnd(rng, (H, D), 0.02), rnd(rng, (D, H), 0.02)
    xn, xc = rnd(rng, (D, S)), rnd(rng, (D, S))
    k = KN.compile_ffn_fused_conv1x1_kern(W1, W3, W2, D, H, S)
    KN.io_write_ffn_fused_conv_input(k, xn, xc)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    k.free()
    h1, h3 = O.sgemm(W1, xn), O.sgemm(W3, xn)  # train_mezo.m:1662-1667 (cpu_only)
    ffn = O.sgemm(W2, (h1 / (1.0 + np.exp(-h1)) * h3).astype(np.float32))
    e = max_rel(y - xc, ffn)  # the W2 projection output (the residual input passes through in fp32)
    print(f"FFN S={S}: max rel err {e:.2e}")
    assert e < TOL, e


def test_lm_head_ce_fp32_inputs(b2p):
    rng = np.random.default_rng(3)
    D, cv, S = 960, 16893, 256
    E, xn = rnd(rng, (cv, D), 0.02), rnd(rng, (D, S))
    tgt = rng.integers(0, cv, S).astype(np.int32)
    k = KN.compile_lm_head_ce_kern(E, D, cv, S)
    k.write(0, xn)
    k.write(1, tgt)
    k.eval()
    loss = float(k.read(0)[0])
    k.free()
    ref = O.cross_entropy(O.sgemm(xn.T.copy(), E.T.copy()), tgt.astype(np.uint16))  # train_mezo.m:1695-1698
    print(f"lm-head CE: |dL| {abs(loss - ref):.2e}")
    assert abs(loss - ref) < 1e-3, (loss, ref)
