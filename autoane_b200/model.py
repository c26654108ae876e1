"""Python mirror of the device-resident MeZO-LoRA-split model (include/b2p.h).

Mirrors the reference's host loop vocabulary (training/train_mezo.m): weights in
LayerWeights layout (fp32 [out, in]), trainable parameters in the
perturb_lora_weights order, channel-first semantics kept at the boundary, and
the MeZO step / data-parallel seed evaluation as single calls into libb2p.so.
Every call runs on the GPU through the C ABI; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib

F16, BF16 = 0, 1
OPT_PAIR_GEMM, OPT_GRAD_SCALE_LOG2, OPT_GRAPHS, OPT_TC_ATTENTION, OPT_TC_ATTENTION_BWD, OPT_PDL = 1, 2, 3, 4, 5, 6


@dataclass
class Config:
    dim: int = 960
    hidden: int = 2560
    heads: int = 15
    kv_heads: int = 5
    head_dim: int = 64
    seq: int = 256
    nlayers: int = 32
    vocab: int = 49152
    rank: int = 8
    rope_theta: float = 100000.0
    res_alpha: float = 1.0
    dtype: int = F16
    max_groups: int = 64
    lora_ffn: bool = False

    def c(self) -> _lib.ModelConfig:
        return _lib.ModelConfig(self.dim, self.hidden, self.heads, self.kv_heads, self.head_dim, self.seq,
                                self.nlayers, self.vocab, self.rank, self.rope_theta, self.res_alpha, self.dtype,
                                self.max_groups, int(self.lora_ffn))


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u16(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


def _u64(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint64))


class Model:
    """A b2p_model on the current CUDA device (call autoane_b200.call('b2p_init', dev) first)."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        self._lib = _lib.load()
        self._cfg_c = cfg.c()
        h = self._lib.b2p_model_create(C.byref(self._cfg_c))
        if not h:
            raise _lib.B2PError("b2p_model_create", -1, self._lib.b2p_last_error().decode())
        self.h = C.c_void_p(h)
        self.P = int(self._lib.b2p_model_trainable_count(self.h))

    def close(self):
        if getattr(self, "h", None):
            self._lib.b2p_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(self._lib.b2p_model_stream(self.h) or 0)

    # ---- weights ----
    def set_layer(self, layer: int, Wq, Wk, Wv, Wo, W1, W2, W3):
        arrs = [np.ascontiguousarray(a, np.float32) for a in (Wq, Wk, Wv, Wo, W1, W2, W3)]
        _lib.call("b2p_model_set_layer", self.h, layer, *[_fp(a) for a in arrs])

    def set_embedding(self, embed, compact_to_full):
        e = np.ascontiguousarray(embed, np.float32)
        c2f = np.ascontiguousarray(compact_to_full, np.int32)
        _lib.call("b2p_model_set_embedding", self.h, _fp(e), c2f.ctypes.data_as(C.POINTER(C.c_int)), len(c2f))

    def set_trainable(self, theta):
        t = np.ascontiguousarray(theta, np.float32)
        _lib.call("b2p_model_set_trainable", self.h, t.ctypes.data, self.P)

    def get_trainable(self) -> np.ndarray:
        out = np.empty(self.P, np.float32)
        _lib.call("b2p_model_get_trainable", self.h, out.ctypes.data, self.P)
        return out

    # ---- evaluation / MeZO ----
    def eval(self, tokens, ctargets, variants) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        vs = (_lib.Variant * len(variants))(*[_lib.Variant(int(s), int(m), float(a), float(b))
                                             for (s, m, a, b) in variants])
        out = np.empty(len(variants), np.float32)
        _lib.call("b2p_model_eval", self.h, _u16(tok), _u16(tgt), n_seq, C.cast(vs, C.c_void_p), len(variants),
                  _fp(out))
        return out

    def group_losses(self, n: int) -> np.ndarray:
        """Per-group losses of the last forward: group g = v * n_seq + q (sequence q, variant v)."""
        out = np.empty(n, np.float32)
        _lib.call("b2p_model_group_losses", self.h, out.ctypes.data, n)
        return out

    def mezo_step(self, tokens, ctargets, seed: int, eps: float, lr: float):
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        lp, lm, g = C.c_float(), C.c_float(), C.c_float()
        _lib.call("b2p_mezo_step", self.h, _u16(tok), _u16(tgt), seed, eps, lr, C.byref(lp), C.byref(lm),
                  C.byref(g))
        return lp.value, lm.value, g.value

    def mezo_eval(self, tokens, ctargets, seeds, eps: float, out=None) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        sd = np.ascontiguousarray(seeds, np.uint64)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        if out is None:
            out = np.empty(2 * len(sd), np.float32)
        ptr = out.ctypes.data if isinstance(out, np.ndarray) else int(out)
        _lib.call("b2p_mezo_eval", self.h, _u16(tok), _u16(tgt), n_seq, _u64(sd), len(sd), eps, ptr)
        return out

    def mezo_eval_device(self, d_tokens: int, d_targets: int, n_seq: int, seeds, eps: float, out_ptr: int):
        """Device-resident inputs (int32 [n_seq, seq] pointers) and a device/host output pointer."""
        sd = np.ascontiguousarray(seeds, np.uint64)
        _lib.call("b2p_mezo_eval_device", self.h, d_tokens, d_targets, n_seq, _u64(sd), len(sd), eps, out_ptr)

    def sync(self):
        _lib.call("b2p_model_sync", self.h)

    def profile(self, enable: bool):
        _lib.call("b2p_model_profile", self.h, int(enable))

    def profile_read(self):
        ms, fl, n = C.c_double(), C.c_double(), C.c_longlong()
        _lib.call("b2p_model_profile_read", self.h, C.byref(ms), C.byref(fl), C.byref(n))
        return ms.value, fl.value, n.value

    def mezo_update(self, seeds, loss_pairs, eps: float, lr: float):
        sd = np.ascontiguousarray(seeds, np.uint64)
        ptr = loss_pairs.ctypes.data if isinstance(loss_pairs, np.ndarray) else int(loss_pairs)
        if isinstance(loss_pairs, np.ndarray):
            assert loss_pairs.dtype == np.float32 and loss_pairs.size >= 2 * len(sd)
        _lib.call("b2p_mezo_update", self.h, _u64(sd), ptr, len(sd), eps, lr)

    def perturb(self, seeds, scales):
        sd = np.ascontiguousarray(seeds, np.uint64)
        sc = np.ascontiguousarray(scales, np.float32)
        _lib.call("b2p_model_perturb", self.h, _u64(sd), _fp(sc), len(sd))

    # ---- backprop-LoRA (P16) ----
    def p16_grad(self, tokens, ctargets):
        """Loss and gradient (trainable layout) of n_seq sequences, parameters unchanged."""
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        loss = C.c_float()
        grad = np.empty(self.P, np.float32)
        _lib.call("b2p_p16_grad", self.h, _u16(tok), _u16(tgt), n_seq, C.byref(loss), grad.ctypes.data)
        return loss.value, grad

    def p16_grad_device(self, d_tokens: int, d_targets: int, n_seq: int, d_loss: int = 0):
        _lib.call("b2p_p16_grad_device", self.h, d_tokens, d_targets, n_seq, d_loss or None)

    def grad_ptr(self) -> int:
        return int(self._lib.b2p_model_grad(self.h) or 0)

    def adam_step(self, lr: float, b1: float = 0.9, b2: float = 0.95, eps: float = 1e-8, wd: float = 0.0):
        _lib.call("b2p_adam_step", self.h, lr, b1, b2, eps, wd)

    def adam_state(self):
        t = C.c_int()
        m = np.empty(self.P, np.float32)
        v = np.empty(self.P, np.float32)
        _lib.call("b2p_adam_state", self.h, 0, C.byref(t), m.ctypes.data, v.ctypes.data)
        return t.value, m, v

    def set_adam_state(self, t: int, m=None, v=None):
        tt = C.c_int(t)
        mm = None if m is None else np.ascontiguousarray(m, np.float32)
        vv = None if v is None else np.ascontiguousarray(v, np.float32)
        _lib.call("b2p_adam_state", self.h, 1, C.byref(tt), None if mm is None else mm.ctypes.data,
                  None if vv is None else vv.ctypes.data)

    def p16_step(self, tokens, ctargets, lr: float) -> float:
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        loss = C.c_float()
        _lib.call("b2p_p16_step", self.h, _u16(tok), _u16(tgt), n_seq, lr, C.byref(loss))
        return loss.value

    # ---- full backprop (train.m) ----
    FULL_WEIGHTS, FULL_WEIGHT_GRADS, FULL_EMBED, FULL_EMBED_GRAD, FULL_TRAINABLE_GRAD = range(5)

    def full_grad(self, tokens, ctargets) -> float:
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        loss = C.c_float()
        _lib.call("b2p_full_grad", self.h, _u16(tok), _u16(tgt), n_seq, C.byref(loss))
        return loss.value

    def full_update(self, lr: float, wd: float = 0.1, clip: float = 1.0) -> float:
        norm = C.c_float()
        _lib.call("b2p_full_update", self.h, lr, wd, clip, C.byref(norm))
        return norm.value

    def full_step(self, tokens, ctargets, lr: float, wd: float = 0.1, clip: float = 1.0):
        tok = np.ascontiguousarray(tokens, np.uint16)
        tgt = np.ascontiguousarray(ctargets, np.uint16)
        n_seq = tok.shape[0] if tok.ndim == 2 else 1
        loss, norm = C.c_float(), C.c_float()
        _lib.call("b2p_full_step", self.h, _u16(tok), _u16(tgt), n_seq, lr, wd, clip, C.byref(loss), C.byref(norm))
        return loss.value, norm.value

    def full_read(self, what: int) -> np.ndarray:
        c = self.cfg
        n = {self.FULL_WEIGHTS: None, self.FULL_WEIGHT_GRADS: None, self.FULL_EMBED: c.vocab * c.dim,
             self.FULL_EMBED_GRAD: c.vocab * c.dim, self.FULL_TRAINABLE_GRAD: self.P}[what]
        if n is None:
            n = int(self._lib.b2p_full_weight_count(self.h))
        out = np.empty(n, np.float32)
        _lib.call("b2p_full_read", self.h, what, out.ctypes.data, n)
        return out

    def split_full_weights(self, flat: np.ndarray) -> dict:
        """Device full-mode layout -> per-layer reference matrices (Wq, Wk, Wv, Wo, W1, W2, W3)."""
        c = self.cfg
        L, D, H = c.nlayers, c.dim, c.hidden
        QD, KVD = c.heads * c.head_dim, c.kv_heads * c.head_dim
        QKV = QD + 2 * KVD
        o = 0
        qkv = flat[o:o + L * QKV * D].reshape(L, QKV, D); o += L * QKV * D
        wo = flat[o:o + L * D * QD].reshape(L, D, QD); o += L * D * QD
        w13 = flat[o:o + L * 2 * H * D].reshape(L, H // 128, 2, 128, D); o += L * 2 * H * D
        w2 = flat[o:o + L * D * H].reshape(L, D, H)
        return {"Wq": [qkv[l, :QD] for l in range(L)], "Wk": [qkv[l, QD:QD + KVD] for l in range(L)],
                "Wv": [qkv[l, QD + KVD:] for l in range(L)], "Wo": [wo[l] for l in range(L)],
                "W1": [w13[l, :, 0].reshape(H, D) for l in range(L)], "W2": [w2[l] for l in range(L)],
                "W3": [w13[l, :, 1].reshape(H, D) for l in range(L)]}

    def set_option(self, option: int, value: int):
        _lib.call("b2p_model_set_option", self.h, option, value)

    # ---- checkpoints (BLZT v4 + LORA sidecar) ----
    def save_checkpoint(self, path, lora_path=None, **header):
        """b2p_ckpt_save; header keywords (step, total_steps, lr, loss, cum_*) fill the CkptHdr."""
        h = _lib.CkptHeader(**header)
        _lib.call("b2p_ckpt_save", self.h, str(path).encode(), None if lora_path is None else str(lora_path).encode(),
                  C.byref(h))

    def load_checkpoint(self, path, lora_path=None, compact_to_full=None, full: bool = False) -> dict:
        """b2p_ckpt_load; returns the file's header as a dict."""
        h = _lib.CkptHeader()
        c2f = None if compact_to_full is None else np.ascontiguousarray(compact_to_full, np.int32)
        _lib.call("b2p_ckpt_load", self.h, str(path).encode(), None if lora_path is None else str(lora_path).encode(),
                  None if c2f is None else c2f.ctypes.data_as(C.POINTER(C.c_int)), 0 if c2f is None else len(c2f),
                  int(full), C.byref(h))
        return header_dict(h)

    def sign_masks(self, seeds) -> np.ndarray:
        sd = np.ascontiguousarray(seeds, np.uint64)
        words = (self.P + 31) // 32
        out = np.empty((len(sd), words), np.uint32)
        _lib.call("b2p_sign_masks", self.h, _u64(sd), len(sd), out.ctypes.data_as(C.POINTER(C.c_uint32)))
        return out


def header_dict(h: _lib.CkptHeader) -> dict:
    return {name: getattr(h, name) for name, _ in h._fields_}


def read_checkpoint_header(path) -> dict:
    """b2p_ckpt_read_header (host only: no device work)."""
    h = _lib.CkptHeader()
    _lib.call("b2p_ckpt_read_header", str(path).encode(), C.byref(h))
    return header_dict(h)


def load_synthetic(model: Model, weights: dict, embed, compact_to_full, theta):
    """Upload reference-layout weights (dict name -> list per layer) into a model."""
    for l in range(model.cfg.nlayers):
        model.set_layer(l, *[weights[k][l] for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")])
    model.set_embedding(embed, compact_to_full)
    model.set_trainable(theta)
