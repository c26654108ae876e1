"""Kern-level operators over the C ABI, with the verbs of the reference's
training/io.h.

`Kern` wraps one `b2p_kernel` (include/b2p.h). The module-level functions keep
the names, argument meaning and channel-first fp32 layout of the reference's
boundary so call sites read the same:

    reference (training/io.h)                        here
    compile_conv1x1_kern(mil, W, ic, oc, seq)   :165  compile_conv1x1_kern(W, ic, oc, seq)
    compile_qkv_fused_conv1x1_kern(...)         :182  compile_qkv_fused_conv1x1_kern(Wq, Wk, Wv, dim, q, kv, seq)
    compile_ffn_fused_conv1x1_kern(...)         :209  compile_ffn_fused_conv1x1_kern(W1, W3, W2, dim, hidden, seq)
    io_write_conv_acts(k->ioIn, act, ic, seq)   :102  io_write_conv_acts(k, act)
    io_write_ffn_fused_conv_input(...)          :232  io_write_ffn_fused_conv_input(k, xnorm, x_cur)
    io_write_dyn(s, act, ic, seq, W, oc)        :79   io_write_dyn(k, act, W)
    ane_eval(k)                                 :242  ane_eval(k)
    io_read_dyn(k->ioOut, out, oc, seq)         :109  io_read_dyn(k) -> [oc, seq]
    free_kern(k)                                :152  free_kern(k)

The MIL text argument has no counterpart: the operator kind is the compile
call. Errors raise `B2PError` (the reference ignores them, io.h:242-249).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (OP_CONV1X1, OP_DX, OP_DYN_MATMUL, OP_FFN_FUSED, OP_LM_HEAD_CE, OP_QKV_FUSED, B2PError,
                   OpDesc)

F16, BF16 = 0, 1


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


class Kern:
    """One compiled operator: weights baked at construction, fp32 channel-first I/O."""

    def __init__(self, kind: int, weights, *, ic: int, seq: int, oc: int = 0, q_dim: int = 0, kv_dim: int = 0,
                 hidden: int = 0, res_alpha: float = 1.0, dtype: int = F16, part_oc=()):
        d = OpDesc()
        d.kind, d.ic, d.oc, d.seq = kind, ic, oc, seq
        d.q_dim, d.kv_dim, d.hidden = q_dim, kv_dim, hidden
        d.res_alpha, d.dtype = res_alpha, dtype
        d.n_parts = len(part_oc)
        for i, v in enumerate(part_oc):
            d.part_oc[i] = v
        self._w = [_f32(w) for w in weights]  # kept alive for the call only; the library copies
        arr = (C.POINTER(C.c_float) * max(1, len(self._w)))(*[_fp(w) for w in self._w])
        lib = _lib.load()
        h = lib.b2p_compile(C.byref(d), arr if self._w else None)
        self._w = None
        if not h:
            raise B2PError("b2p_compile", -1, lib.b2p_last_error().decode(errors="replace"))
        self.h = h
        self.desc = d

    # -- I/O ------------------------------------------------------------
    def input_shape(self, idx: int):
        n = _lib.load().b2p_input_bytes(self.h, idx) // 4
        return n

    def write(self, idx: int, data) -> None:
        if self.desc.kind == OP_LM_HEAD_CE and idx == 1:
            a = np.ascontiguousarray(data, dtype=np.int32)
        else:
            a = _f32(data)
        _lib.call("b2p_write_input", self.h, idx, a.ctypes.data_as(C.c_void_p), a.nbytes)

    def write_channels(self, idx: int, ch_off: int, data) -> None:
        a = _f32(data)
        _lib.call("b2p_write_input_channels", self.h, idx, ch_off, a.shape[0], _fp(a))

    def eval(self) -> None:
        _lib.call("b2p_eval", self.h)

    def eval_async(self) -> None:
        _lib.call("b2p_eval_async", self.h)

    def read(self, idx: int = 0) -> np.ndarray:
        n = _lib.load().b2p_output_bytes(self.h, idx)
        out = np.empty(n // 4, np.float32)
        _lib.call("b2p_read_output", self.h, idx, _fp(out), n)
        return out

    def read_channels(self, idx: int, ch_off: int, channels: int) -> np.ndarray:
        S = 1 if self.desc.kind == OP_LM_HEAD_CE else self.desc.seq
        out = np.empty((channels, S), np.float32)
        _lib.call("b2p_read_output_channels", self.h, idx, ch_off, channels, _fp(out))
        return out

    # -- device-resident extensions --------------------------------------
    def set_lora(self, part: int, A, B, rank: int | None = None) -> None:
        if A is None and B is None:
            _lib.call("b2p_set_lora", self.h, part, None, None, 0)
            return
        A, B = _f32(A), _f32(B)
        _lib.call("b2p_set_lora", self.h, part, _fp(A), _fp(B), rank or A.shape[0])

    def set_perturb(self, seed: int, scale: float) -> None:
        _lib.call("b2p_set_perturb", self.h, C.c_uint64(seed), np.float32(scale))

    def free(self) -> None:
        if self.h:
            _lib.load().b2p_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---- io.h verbs ---------------------------------------------------------
def compile_conv1x1_kern(W, ic: int, oc: int, seq: int, dtype: int = F16) -> Kern:
    return Kern(OP_CONV1X1, [W], ic=ic, oc=oc, seq=seq, dtype=dtype)


def compile_qkv_fused_conv1x1_kern(Wq, Wk, Wv, dim: int, q_dim: int, kv_dim: int, seq: int,
                                   dtype: int = F16) -> Kern:
    return Kern(OP_QKV_FUSED, [Wq, Wk, Wv], ic=dim, seq=seq, q_dim=q_dim, kv_dim=kv_dim, dtype=dtype)


def compile_ffn_fused_conv1x1_kern(W1, W3, W2, dim: int, hidden: int, seq: int, res_alpha: float = 1.0,
                                   dtype: int = F16) -> Kern:
    return Kern(OP_FFN_FUSED, [W1, W3, W2], ic=dim, seq=seq, hidden=hidden, res_alpha=res_alpha, dtype=dtype)


def compile_dyn_matmul_kern(ic: int, oc: int, seq: int, dtype: int = F16) -> Kern:
    return Kern(OP_DYN_MATMUL, [], ic=ic, oc=oc, seq=seq, dtype=dtype)


def compile_lm_head_ce_kern(cembed, dim: int, cv: int, seq: int, dtype: int = F16) -> Kern:
    return Kern(OP_LM_HEAD_CE, [cembed], ic=dim, oc=cv, seq=seq, dtype=dtype)


def compile_dx_kern(weights, ic: int, seq: int, dtype: int = F16) -> Kern:
    """dx = sum_i W_i^T · dy_i for W_i [oc_i, ic] (the backward data GEMMs)."""
    ws = [_f32(w) for w in weights]
    return Kern(OP_DX, ws, ic=ic, seq=seq, dtype=dtype, part_oc=[w.shape[0] for w in ws])


def io_write_conv_acts(k: Kern, act) -> None:
    k.write(0, act)


def io_write_ffn_fused_conv_input(k: Kern, xnorm, x_cur) -> None:
    k.write(0, xnorm)
    k.write(1, x_cur)


def io_write_dyn(k: Kern, act, W) -> None:
    k.write(0, act)
    k.write(1, W)


def io_write_dyn_acts(k: Kern, act) -> None:
    k.write(0, act)


def ane_eval(k: Kern) -> None:
    k.eval()


def io_read_dyn(k: Kern) -> np.ndarray:
    d = k.desc
    C_ = {OP_CONV1X1: d.oc, OP_DYN_MATMUL: d.oc, OP_QKV_FUSED: d.q_dim + 2 * d.kv_dim, OP_FFN_FUSED: d.ic,
          OP_DX: d.ic, OP_LM_HEAD_CE: 1}[d.kind]
    S = 1 if d.kind == OP_LM_HEAD_CE else d.seq
    return k.read(0).reshape(C_, S)


def free_kern(k: Kern) -> None:
    k.free()


def compile_count() -> int:
    return _lib.load().b2p_compile_count()


def reset_compile_count() -> None:
    _lib.load().b2p_reset_compile_count()
