"""Kern-level operators (b2p_compile / write / eval / read) against the oracle.

The oracle restates the reference's CPU path for each operator (cblas_sgemm
projections, lora_addmm, cross_entropy_loss). The device computes from 16-bit
operands, as the reference's Neural-Engine path does after cvt_f32_f16 on
write (training/io.h:42-51, :102), so the oracle is fed the same fp16-rounded
inputs and the remaining difference is fp32 accumulation order plus the 16-bit
intermediates named in each test. Tolerances are relative to the output's
largest magnitude:
  * plain projections (fp32 accumulate, fp32 out): 1e-5
  * LoRA (16-bit A·x and perturbed B operands):    2e-3
  * FFN (16-bit gate between the two GEMMs):       1e-3 (measured 8e-5 - 1.2e-4)
  * cross-entropy: |ΔL| < 1e-3 nats
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from autoane_b200 import kern as KN
from autoane_b200._lib import B2PError
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def h16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def rnd(rng, shape, std=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)


def close(got, ref, rel):
    err = np.max(np.abs(got - ref))
    scale = max(np.max(np.abs(ref)), 1e-6)
    print(f"max rel err {err / scale:.2e} (gate {rel})")
    assert err <= rel * scale, f"max err {err:.3e} vs scale {scale:.3e} (rel {err / scale:.2e} > {rel})"


@pytest.mark.parametrize("ic,oc,S", [(960, 320, 256), (960, 960, 128), (2560, 960, 512), (64, 8, 64), (72, 200, 300)])
def test_conv1x1_matches_sgemm(b2p, ic, oc, S):
    rng = np.random.default_rng(ic + oc + S)
    W, x = rnd(rng, (oc, ic), 0.02), rnd(rng, (ic, S))
    k = KN.compile_conv1x1_kern(W, ic, oc, S)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    close(y, O.sgemm(h16(W), h16(x)), 1e-5)
    KN.free_kern(k)


def test_qkv_fused_concat_matches_sgemm(b2p):
    rng = np.random.default_rng(3)
    D, Q, KV, S = 960, 960, 320, 256
    Wq, Wk, Wv = rnd(rng, (Q, D), 0.02), rnd(rng, (KV, D), 0.02), rnd(rng, (KV, D), 0.02)
    x = rnd(rng, (D, S))
    k = KN.compile_qkv_fused_conv1x1_kern(Wq, Wk, Wv, D, Q, KV, S)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    assert y.shape == (Q + 2 * KV, S)
    xr = h16(x)
    close(y[:Q], O.sgemm(h16(Wq), xr), 1e-5)
    close(y[Q:Q + KV], O.sgemm(h16(Wk), xr), 1e-5)
    close(y[Q + KV:], O.sgemm(h16(Wv), xr), 1e-5)
    # channel-range read (io_read_fp16 with a channel offset)
    close(k.read_channels(0, Q, KV), y[Q:Q + KV], 0.0)
    k.free()


def _lora_params(rng, parts, D, r):
    return [(rnd(rng, (r, D), 1.0 / np.sqrt(r)), rnd(rng, (o, r), 0.01)) for o in parts]


def _perturbed(params, seed, scale):
    """Adapters after perturb_buffer over A_0, B_0, A_1, B_1, ... with one stream (train_mezo.m:122-136)."""
    flat = np.concatenate([np.concatenate([A.ravel(), B.ravel()]) for A, B in params]).astype(np.float32)
    sizes = [n for A, B in params for n in (A.size, B.size)]
    mask = O.sign_mask(seed, sizes)
    bits = (mask[np.arange(flat.size) >> 5] >> (np.arange(flat.size) & 31)) & 1
    s = np.float32(scale)
    flat = (flat + np.where(bits == 1, s, -s).astype(np.float32)).astype(np.float32)
    out, o = [], 0
    for A, B in params:
        a = flat[o:o + A.size].reshape(A.shape); o += A.size
        b = flat[o:o + B.size].reshape(B.shape); o += B.size
        out.append((a, b))
    return out


@pytest.mark.parametrize("rank", [8, 4])
@pytest.mark.parametrize("seed,scale", [(0, 0.0), (7 * 1000003 + 42, 0.05), (12345, -0.1)])
def test_qkv_fused_lora_and_perturbation(b2p, rank, seed, scale):
    rng = np.random.default_rng(rank * 100 + seed % 97)
    D, Q, KV, S = 960, 960, 320, 256
    Ws = [rnd(rng, (o, D), 0.02) for o in (Q, KV, KV)]
    x = rnd(rng, (D, S))
    params = _lora_params(rng, (Q, KV, KV), D, rank)
    k = KN.compile_qkv_fused_conv1x1_kern(*Ws, D, Q, KV, S)
    for i, (A, B) in enumerate(params):
        k.set_lora(i, A, B, rank)
    k.set_perturb(seed, scale)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    use = _perturbed(params, seed, scale) if scale else params
    xr = h16(x)
    row = 0
    for W, (A, B), o in zip(Ws, use, (Q, KV, KV)):
        ref = O.sgemm(h16(W), xr)
        O.lora_addmm(ref, A, B, xr)  # the conv-fused path's host-side adapter (train_mezo.m:1558-1560)
        close(y[row:row + o], ref, 2e-3)
        row += o
    # the stored adapters are untouched: turning the perturbation off restores the unperturbed result
    k.set_perturb(seed, 0.0)
    KN.ane_eval(k)
    y0 = KN.io_read_dyn(k)
    ref0 = O.sgemm(h16(Ws[0]), xr)
    O.lora_addmm(ref0, *params[0], xr)
    close(y0[:Q], ref0, 2e-3)
    if scale:  # and the perturbation is large enough to be seen at this tolerance
        assert np.max(np.abs(y[:Q] - y0[:Q])) > 10 * 2e-3 * np.max(np.abs(ref0))
    k.free()


def test_conv1x1_lora_removal_and_partial_parts(b2p):
    rng = np.random.default_rng(11)
    D, S = 960, 256
    W, x = rnd(rng, (D, D), 0.02), rnd(rng, (D, S))
    A, B = rnd(rng, (8, D), 0.35), rnd(rng, (D, 8), 0.01)
    k = KN.compile_conv1x1_kern(W, D, D, S)
    k.set_lora(0, A, B)
    KN.io_write_conv_acts(k, x)
    KN.ane_eval(k)
    ref = O.sgemm(h16(W), h16(x))
    with_lora = ref.copy()
    O.lora_addmm(with_lora, A, B, h16(x))
    close(KN.io_read_dyn(k), with_lora, 2e-3)
    k.set_lora(0, None, None)
    KN.ane_eval(k)
    close(KN.io_read_dyn(k), ref, 1e-5)
    k.free()
    # qkv with only some parts carrying adapters is refused at eval
    q = KN.compile_qkv_fused_conv1x1_kern(W, W[:320], W[:320], D, D, 320, S)
    q.set_lora(0, A, B)
    KN.io_write_conv_acts(q, x)
    with pytest.raises(B2PError, match="set all or none"):
        KN.ane_eval(q)
    q.free()


@pytest.mark.parametrize("S,alpha", [(256, 1.0), (128, 0.5), (512, 1.0)])
def test_ffn_fused_matches_oracle(b2p, S, alpha):
    rng = np.random.default_rng(S)
    D, H = 960, 2560
    W1, W3, W2 = rnd(rng, (H, D), 0.02), rnd(rng, (H, D), 0.02), rnd(rng, (D, H), 0.02)
    xn, xc = rnd(rng, (D, S)), rnd(rng, (D, S))
    k = KN.compile_ffn_fused_conv1x1_kern(W1, W3, W2, D, H, S, res_alpha=alpha)
    KN.io_write_ffn_fused_conv_input(k, xn, xc)
    KN.ane_eval(k)
    y = KN.io_read_dyn(k)
    # mil_dynamic.h:82-131: x_next = x_cur + alpha·W2(silu(W1 xn) ⊙ W3 xn)
    h1, h3 = O.sgemm(h16(W1), h16(xn)), O.sgemm(h16(W3), h16(xn))
    gate = h16(h1 / (1.0 + np.exp(-h1)) * h3)
    ref = (xc + np.float32(alpha) * O.sgemm(h16(W2), gate)).astype(np.float32)
    close(y - xc, ref - xc, 1e-3)
    # eval is repeatable: the residual input is not consumed
    KN.ane_eval(k)
    close(KN.io_read_dyn(k), y, 0.0)
    k.free()


@pytest.mark.parametrize("ic,oc,S", [(960, 320, 256), (256, 1024, 128)])
def test_dyn_matmul_matches_sgemm(b2p, ic, oc, S):
    rng = np.random.default_rng(oc)
    act, W = rnd(rng, (ic, S)), rnd(rng, (ic, oc), 0.02)
    k = KN.compile_dyn_matmul_kern(ic, oc, S)
    KN.io_write_dyn(k, act, W)
    KN.ane_eval(k)
    # gen_dyn_matmul (mil_dynamic.h:133-155): y = (act^T · W)^T
    close(KN.io_read_dyn(k), O.sgemm(h16(W).T, h16(act)), 1e-5)
    # new activations with the weights already staged (io_write_dyn_acts, io.h:92)
    act2 = rnd(rng, (ic, S))
    KN.io_write_dyn_acts(k, act2)
    KN.ane_eval(k)
    close(KN.io_read_dyn(k), O.sgemm(h16(W).T, h16(act2)), 1e-5)
    k.free()


@pytest.mark.parametrize("cv,S", [(16893, 256), (1000, 128)])
def test_lm_head_ce_matches_oracle(b2p, cv, S):
    rng = np.random.default_rng(cv)
    D = 960
    E, xn = rnd(rng, (cv, D), 0.02), rnd(rng, (D, S))
    tgt = rng.integers(0, cv, S).astype(np.int32)
    k = KN.compile_lm_head_ce_kern(E, D, cv, S)
    k.write(0, xn)
    k.write(1, tgt)
    k.eval()
    loss = float(k.read(0)[0])
    logits = O.sgemm(h16(xn).T, h16(E).T)  # token-major [S, CV] (train_mezo.m:1695-1698)
    ref = O.cross_entropy(logits, tgt.astype(np.uint16))
    assert abs(loss - ref) < 1e-3, (loss, ref)
    bad = tgt.copy()
    bad[3] = cv
    with pytest.raises(B2PError, match="outside"):
        k.write(1, bad)
    k.free()


def test_dx_sums_transposed_parts(b2p):
    rng = np.random.default_rng(5)
    D, H, S = 960, 2560, 256
    W1, W3 = rnd(rng, (H, D), 0.02), rnd(rng, (H, D), 0.02)
    dh1, dh3 = rnd(rng, (H, S)), rnd(rng, (H, S))
    k = KN.compile_dx_kern([W1, W3], D, S)
    k.write(0, dh1)
    k.write(1, dh3)
    k.eval()
    got = k.read(0).reshape(D, S)
    # ffnBwdW13t (mil_dynamic.h:420): dx = W1^T dh1 + W3^T dh3
    ref = O.sgemm(h16(W1).T, h16(dh1)) + O.sgemm(h16(W3).T, h16(dh3))
    close(got, ref, 1e-5)
    k.free()


def test_write_channels_and_bounds(b2p):
    rng = np.random.default_rng(9)
    D, S = 960, 128
    W, x = rnd(rng, (320, D), 0.02), rnd(rng, (D, S))
    k = KN.compile_conv1x1_kern(W, D, 320, S)
    k.write_channels(0, 0, x[:500])
    k.write_channels(0, 500, x[500:])  # io_write_fp16_at (io.h:72)
    k.eval()
    close(KN.io_read_dyn(k), O.sgemm(h16(W), h16(x)), 1e-5)
    with pytest.raises(B2PError, match="out of range"):
        k.write(1, x)
    with pytest.raises(B2PError, match="bytes"):
        k.write(0, x[:, :64])
    with pytest.raises(B2PError, match="outside"):
        k.write_channels(0, 900, x[:100])
    with pytest.raises(B2PError, match="out of range"):
        k.read(1)
    k.free()


def test_compile_count_and_bad_descriptors(b2p):
    KN.reset_compile_count()
    rng = np.random.default_rng(1)
    W = rnd(rng, (64, 64), 0.02)
    ks = [KN.compile_conv1x1_kern(W, 64, 64, 128) for _ in range(3)]
    assert KN.compile_count() == 3
    for k in ks:
        k.free()
    with pytest.raises(B2PError, match="multiple of 8"):
        KN.compile_conv1x1_kern(rnd(rng, (60, 64)), 64, 60, 128)
    with pytest.raises(B2PError, match="hidden"):
        KN.compile_ffn_fused_conv1x1_kern(W, W, W, 64, 100, 128)
    assert KN.compile_count() == 3


def test_io_shim_call_site_compiles_and_matches(b2p, tmp_path):
    """A C call site written against io.h's names, built with include/b2p_io.h in its place."""
    so = tmp_path / "site.so"
    subprocess.run(["gcc", "-std=c11", "-O2", "-shared", "-fPIC", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "shim" / "conv_fused_site.c"), "-o", str(so),
                    "-L", str(ROOT / "autoane_b200"), "-lb2p", f"-Wl,-rpath,{ROOT / 'autoane_b200'}"],
                   check=True)
    lib = C.CDLL(str(so))
    rng = np.random.default_rng(21)
    D, Q, KV, H, S = 960, 960, 320, 2560, 256
    w = {n: rnd(rng, s, 0.02) for n, s in (("Wq", (Q, D)), ("Wk", (KV, D)), ("Wv", (KV, D)), ("Wo", (D, Q)),
                                           ("W1", (H, D)), ("W2", (D, H)), ("W3", (H, D)))}
    xn, attn, x2n, xc = rnd(rng, (D, S)), rnd(rng, (Q, S)), rnd(rng, (D, S)), rnd(rng, (D, S))
    x_io = xc.copy()
    Qo, Ko, Vo, oo = (np.zeros((c, S), np.float32) for c in (Q, KV, KV, D))
    fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))
    rc = lib.site_layer(*[fp(w[n]) for n in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")], D, Q, KV, H, S,
                        fp(xn), fp(attn), fp(x2n), fp(x_io), fp(Qo), fp(Ko), fp(Vo), fp(oo))
    assert rc == 0
    # outputs pass through the fp16 surface, as IOSurface reads do (io.h:58-61)
    close(Qo, O.sgemm(h16(w["Wq"]), h16(xn)), 1e-3)
    close(Ko, O.sgemm(h16(w["Wk"]), h16(xn)), 1e-3)
    close(Vo, O.sgemm(h16(w["Wv"]), h16(xn)), 1e-3)
    close(oo, O.sgemm(h16(w["Wo"]), h16(attn)), 1e-3)
    h1, h3 = O.sgemm(h16(w["W1"]), h16(x2n)), O.sgemm(h16(w["W3"]), h16(x2n))
    ffn = O.sgemm(h16(w["W2"]), h16(h1 / (1.0 + np.exp(-h1)) * h3))
    # x_cur comes back through the fp16 surface (io_read_dyn, io.h:109-114): every element
    # is the fp16 rounding of x + FFN(x), so it may differ from the rounded oracle value by
    # one fp16 ulp plus the FFN's own error (gated at 1e-3 of its largest value, as above)
    ref16 = h16(h16(xc) + ffn)
    ulp = np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float32)
    bound = ulp + 1e-3 * np.max(np.abs(ffn))
    assert np.all(np.abs(x_io - ref16) <= bound), np.max(np.abs(x_io - ref16) / bound)


def test_io_shim_dyn_matmul_requests_compile_and_match(b2p, tmp_path):
    """compile_kern_mil_w / io_write_dyn / make_request / ane_eval_req / io_write_dyn_acts from C."""
    so = tmp_path / "dyn.so"
    subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", "-I",
                    str(ROOT / "include"), str(ROOT / "tests" / "shim" / "dyn_site.c"), "-o", str(so),
                    "-L", str(ROOT / "autoane_b200"), "-lb2p", f"-Wl,-rpath,{ROOT / 'autoane_b200'}"], check=True)
    lib = C.CDLL(str(so))
    rng = np.random.default_rng(23)
    ic, oc, S = 960, 320, 256
    a1, a2, a3 = rnd(rng, (ic, S)), rnd(rng, (ic, S)), rnd(rng, (ic, S))
    w1, w2 = rnd(rng, (ic, oc), 0.02), rnd(rng, (ic, oc), 0.02)
    out = np.zeros((4, oc, S), np.float32)
    fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    assert lib.site_dyn(fp(a1), fp(w1), fp(a2), fp(w2), fp(a3), ic, oc, S, fp(out)) == 0
    # results pass through the fp16 output surface (io.h:109-114)
    for got, (w, a) in zip(out, ((w1, a1), (w2, a2), (w2, a3), (w1, a1))):
        close(got, h16(O.sgemm(h16(w).T, h16(a))), 1e-3)
