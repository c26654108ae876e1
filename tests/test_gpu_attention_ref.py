"""Attention forward and backward on the device (b2p_attention / b2p_attention_backward,
the kernels the model and the backprop-LoRA backward run) against the reference's own
compiled code: cpu_sdpa_forward and cpu_sdpa_backward (training/cpu_ops.h:213-360)
with the GQA tiling / reduction and inverse RoPE that bp_lora_backward applies
around them (training/backprop_lora.h:241-252), from oracle/_ref.

Inputs are fp16-representable, so both sides see the same Q, K, V and dO. The
device keeps P, dS and its outputs in 16 bit with fp32 accumulation; the tolerance
is normwise relative L2 per tensor (||dev - ref|| / ||ref||):
  * forward output O: < 1e-3 (16-bit P and O: unit roundoff 4.9e-4, averaged over
    up to 256 keys; measured 2.3e-4);
  * dV, dK, dQ: < 2e-3 (16-bit P and dS operands of four chained products, and
    the dS = P·(dP - D) cancellation, which grows the relative error of small dS
    entries; measured 2.9-3.9e-4; a wrong term in any one product fails by far).
Cases: SmolLM2-360M heads (15 query / 5 KV, theta 100000) at 256 and 128 tokens, fp16,
over 3 sequences (tcgen05 kernels), plus one bf16 case at < 5e-3 / 1e-2 (8-bit mantissa;
measured 1.8e-3 / 3.0e-3).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from autoane_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

F = C.POINTER(C.c_float)
HD = 64


def f(a):
    return a.ctypes.data_as(F)


def ref_attention(ref, Q, K, V, dA, heads, kv_heads, seq):
    """One sequence, channel-first [C, seq] fp32; returns O, dQ, dK, dV (dQ/dK pre-RoPE)."""
    g = heads // kv_heads
    kt = np.ascontiguousarray(np.repeat(K.reshape(kv_heads, HD, seq), g, axis=0).reshape(heads * HD, seq))
    vt = np.ascontiguousarray(np.repeat(V.reshape(kv_heads, HD, seq), g, axis=0).reshape(heads * HD, seq))
    o = np.zeros((heads * HD, seq), np.float32)
    ref.ref_sdpa_forward(f(Q), f(kt), f(vt), f(o), heads, HD, seq)
    dq, dkf, dvf = (np.zeros((heads * HD, seq), np.float32) for _ in range(3))
    ref.ref_sdpa_backward(f(Q), f(kt), f(vt), f(dA), f(dq), f(dkf), f(dvf), heads, HD, seq)
    dk = np.ascontiguousarray(dkf.reshape(kv_heads, g, HD, seq).sum(axis=1).reshape(kv_heads * HD, seq))
    dv = np.ascontiguousarray(dvf.reshape(kv_heads, g, HD, seq).sum(axis=1).reshape(kv_heads * HD, seq))
    ref.ref_rope_backward(f(dq), seq, heads * HD, HD)
    ref.ref_rope_backward(f(dk), seq, kv_heads * HD, HD)
    return o, dq, dk, dv


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


@pytest.mark.parametrize("seq,dtype,tol_o,tol_g", [(256, 0, 1e-3, 2e-3), (128, 0, 1e-3, 2e-3),
                                                   (256, 1, 5e-3, 1e-2)],
                         ids=["seq256_f16", "seq128_f16", "seq256_bf16"])
def test_attention_matches_reference_sdpa(b2p, seq, dtype, tol_o, tol_g):
    ref = O.ref_lib("smollm2_360m")  # ROPE_THETA 100000 compiled in (training/models/smollm2_360m.h)
    if ref is None:
        pytest.skip("oracle/_ref not built")
    heads, kv, nseq = 15, 5, 3
    QD, KVD = heads * HD, kv * HD
    W = QD + 2 * KVD
    rng = np.random.default_rng(seq + dtype)
    tdt = torch.bfloat16 if dtype else torch.float16
    # post-RoPE Q, K and V at the scale of the model's projections; dO at the scale of dL/dO
    qkv = torch.tensor(rng.standard_normal((nseq * seq, W), dtype=np.float32) * 1.5).to(tdt)
    dout = torch.tensor(rng.standard_normal((nseq * seq, QD), dtype=np.float32) * 1e-2).to(tdt)
    d_qkv, d_dout = qkv.cuda(), dout.cuda()
    d_out = torch.zeros((nseq * seq, QD), dtype=tdt, device="cuda")
    d_lse = torch.zeros((nseq * seq, heads), dtype=torch.float32, device="cuda")
    d_dqkv = torch.zeros((nseq * seq, W), dtype=tdt, device="cuda")
    _lib.call("b2p_attention", d_qkv.data_ptr(), W, d_out.data_ptr(), QD, d_lse.data_ptr(), nseq, seq, heads, kv,
              dtype, None)
    _lib.call("b2p_attention_backward", d_qkv.data_ptr(), W, d_out.data_ptr(), d_dout.data_ptr(), QD,
              d_lse.data_ptr(), d_dqkv.data_ptr(), W, nseq, seq, heads, kv, 100000.0, dtype, None)
    torch.cuda.synchronize()
    _lib.call("b2p_device_status", None)
    q32, do32 = qkv.float().numpy(), dout.float().numpy()
    out, dqkv = d_out.float().cpu().numpy(), d_dqkv.float().cpu().numpy()
    worst = {}
    for s in range(nseq):
        rows = slice(s * seq, (s + 1) * seq)
        cf = lambda a: np.ascontiguousarray(a.T)  # token-major -> channel-first  # noqa: E731
        Q, K, V = cf(q32[rows, :QD]), cf(q32[rows, QD:QD + KVD]), cf(q32[rows, QD + KVD:])
        o, dq, dk, dv = ref_attention(ref, Q, K, V, cf(do32[rows]), heads, kv, seq)
        got = {"O": cf(out[rows]), "dQ": cf(dqkv[rows, :QD]), "dK": cf(dqkv[rows, QD:QD + KVD]),
               "dV": cf(dqkv[rows, QD + KVD:])}
        for name, r in (("O", o), ("dQ", dq), ("dK", dk), ("dV", dv)):
            worst[name] = max(worst.get(name, 0.0), rel(got[name], r))
    print(f"attention vs reference cpu_sdpa (seq {seq}, dtype {dtype}): " +
          ", ".join(f"{k} {v:.2e}" for k, v in worst.items()))
    assert worst["O"] < tol_o, worst
    for name in ("dQ", "dK", "dV"):
        assert worst[name] < tol_g, worst
