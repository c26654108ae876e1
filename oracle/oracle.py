"""ctypes wrapper of oracle/liboracle.so and oracle/_ref/libref_*.so.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker. The product (libb2p.so) never
calls it.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_lib = None


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u16(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


class Layout(C.Structure):
    _fields_ = [(n, C.c_int64) for n in
                ("Aq", "Bq", "Ak", "Bk", "Av", "Bv", "Ao", "Bo", "rms_att", "rms_ffn", "layer_size", "rms_final",
                 "total", "A1", "B1", "A2", "B2", "A3", "B3")]


class _Model(C.Structure):
    _fields_ = ([(n, C.c_int) for n in ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers", "vocab",
                                         "cv", "rank")]
                + [("rope_theta", C.c_float), ("res_alpha", C.c_float)]
                + [(n, C.POINTER(C.POINTER(C.c_float))) for n in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")]
                + [("embed", C.POINTER(C.c_float)), ("cembed", C.POINTER(C.c_float))]
                + [("lora_ffn", C.c_int)])


class _Taps(C.Structure):
    _fields_ = [(n, C.POINTER(C.c_float)) for n in ("x_final", "xn_final", "logits", "layer_x")]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        p = HERE / "liboracle.so"
        if not p.exists():
            from . import build as _b  # type: ignore
            _b.build_oracle()
        L = C.CDLL(str(p))
        L.or_xo_next.restype = C.c_uint64
        L.or_xo_seed.argtypes = [C.c_void_p, C.c_uint64]
        L.or_xo_next.argtypes = [C.c_void_p]
        L.or_perturb_buffer.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_size_t, C.c_float]
        L.or_sign_mask.argtypes = [C.c_uint64, C.POINTER(C.c_int64), C.c_int, C.POINTER(C.c_uint32)]
        L.or_lora_layout.restype = Layout
        L.or_lora_layout.argtypes = [C.c_int] * 5
        L.or_perturb_lora.argtypes = [C.POINTER(C.c_float)] + [C.c_int] * 5 + [C.c_uint64, C.c_float]
        L.or_lora_buffer_sizes.argtypes = [C.c_int] * 5 + [C.POINTER(C.c_int64)]
        L.or_lora_layout_ffn.restype = Layout
        L.or_lora_layout_ffn.argtypes = [C.c_int] * 7
        L.or_lora_buffer_sizes_ffn.argtypes = [C.c_int] * 7 + [C.POINTER(C.c_int64)]
        L.or_perturb_lora_ffn.argtypes = [C.POINTER(C.c_float)] + [C.c_int] * 7 + [C.c_uint64, C.c_float]
        L.or_forward_loss.restype = C.c_float
        L.or_forward_loss.argtypes = [C.POINTER(_Model), C.POINTER(C.c_float), C.POINTER(C.c_uint16),
                                      C.POINTER(C.c_uint16), C.POINTER(_Taps)]
        L.or_mezo_step.argtypes = [C.POINTER(_Model), C.POINTER(C.c_float), C.POINTER(C.c_uint16),
                                   C.POINTER(C.c_uint16), C.c_uint64, C.c_float, C.c_float,
                                   C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.or_rope_tables.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_int, C.c_int, C.c_float]
        L.or_set_threads.argtypes = [C.c_int]
        L.or_set_threads.restype = C.c_int
        L.or_cross_entropy.restype = C.c_float
        L.or_cross_entropy.argtypes = [C.POINTER(C.c_float), C.POINTER(C.c_uint16), C.c_int, C.c_int]
        L.or_lora_addmm.argtypes = [C.POINTER(C.c_float)] * 5 + [C.c_int] * 4
        L.or_p16_grad.restype = C.c_float
        L.or_p16_grad.argtypes = [C.POINTER(_Model), C.POINTER(C.c_float), C.POINTER(C.c_uint16),
                                  C.POINTER(C.c_uint16), C.POINTER(C.c_float)]
        L.or_full_grad.restype = C.c_float
        L.or_full_grad.argtypes = [C.POINTER(_Model), C.POINTER(C.c_float), C.POINTER(C.c_uint16),
                                   C.POINTER(C.c_uint16), C.POINTER(C.c_float), C.POINTER(C.c_float),
                                   C.POINTER(C.c_float), C.POINTER(C.c_int32)]
        L.or_adam.argtypes = [C.POINTER(C.c_float)] * 4 + [C.c_size_t, C.c_int] + [C.c_float] * 5
        L.or_sgemm_nn.argtypes = [C.c_int] * 3 + [C.POINTER(C.c_float)] * 3 + [C.c_float]
        for n in ("or_rmsnorm",):
            getattr(L, n).argtypes = [C.POINTER(C.c_float)] * 3 + [C.c_int, C.c_int]
        L.or_rope_forward.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_float]
        L.or_sdpa_forward.argtypes = [C.POINTER(C.c_float)] * 4 + [C.c_int] * 3
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    return lib().or_set_threads(n)


# ---------------- PRNG / perturbation ----------------
def xo_draws(seed: int, n: int) -> list[int]:
    st = (C.c_uint64 * 4)()
    lib().or_xo_seed(st, seed)
    return [lib().or_xo_next(st) for _ in range(n)]


def perturb_buffer(seed: int, buf: np.ndarray, scale: float) -> None:
    """Seed a fresh stream and apply perturb_buffer to one float32 buffer in place."""
    assert buf.dtype == np.float32 and buf.flags.c_contiguous
    st = (C.c_uint64 * 4)()
    lib().or_xo_seed(st, seed)
    lib().or_perturb_buffer(st, _f(buf), C.c_size_t(buf.size), C.c_float(np.float32(scale)))


def sign_mask(seed: int, sizes) -> np.ndarray:
    sizes = np.ascontiguousarray(sizes, dtype=np.int64)
    total = int(sizes.sum())
    out = np.zeros((total + 31) // 32, dtype=np.uint32)
    lib().or_sign_mask(seed, sizes.ctypes.data_as(C.POINTER(C.c_int64)), len(sizes),
                       out.ctypes.data_as(C.POINTER(C.c_uint32)))
    return out


def lora_layout(nlayers, dim, q_dim, kv_dim, rank) -> Layout:
    return lib().or_lora_layout(nlayers, dim, q_dim, kv_dim, rank)


def lora_layout_ffn(nlayers, dim, q_dim, kv_dim, hidden, rank, ffn) -> Layout:
    """or_lora_layout_ffn: the layout with the --lora-ffn adapters after Bo (train_mezo.m:575-582)."""
    return lib().or_lora_layout_ffn(nlayers, dim, q_dim, kv_dim, hidden, rank, int(ffn))


def lora_buffer_sizes_ffn(nlayers, dim, q_dim, kv_dim, hidden, rank, ffn) -> np.ndarray:
    out = np.zeros(16 * nlayers + 1, np.int64)
    n = lib().or_lora_buffer_sizes_ffn(nlayers, dim, q_dim, kv_dim, hidden, rank, int(ffn),
                                       out.ctypes.data_as(C.POINTER(C.c_int64)))
    return out[:n]


def perturb_lora_ffn(theta: np.ndarray, nlayers, dim, q_dim, kv_dim, hidden, rank, ffn, seed: int,
                     scale: float) -> None:
    assert theta.dtype == np.float32 and theta.flags.c_contiguous
    lib().or_perturb_lora_ffn(_f(theta), nlayers, dim, q_dim, kv_dim, hidden, rank, int(ffn), seed,
                              np.float32(scale))


def lora_buffer_sizes(nlayers, dim, q_dim, kv_dim, rank) -> np.ndarray:
    out = np.zeros(10 * nlayers + 1, dtype=np.int64)
    n = lib().or_lora_buffer_sizes(nlayers, dim, q_dim, kv_dim, rank, out.ctypes.data_as(C.POINTER(C.c_int64)))
    return out[:n]


def perturb_lora(theta: np.ndarray, nlayers, dim, q_dim, kv_dim, rank, seed: int, scale: float) -> None:
    assert theta.dtype == np.float32 and theta.flags.c_contiguous
    lib().or_perturb_lora(_f(theta), nlayers, dim, q_dim, kv_dim, rank, seed, np.float32(scale))


def sgemm(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """C = A·B in fp32 through cblas_sgemm (the reference's projection call sites)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    out = np.zeros((M, N), np.float32)
    lib().or_sgemm_nn(M, N, K, _f(A), _f(B), _f(out), np.float32(0.0))
    return out


def lora_addmm(out: np.ndarray, A: np.ndarray, B: np.ndarray, x: np.ndarray) -> None:
    """out[out_dim, S] += B·(A·x) in place (lora_addmm, training/train_mezo.m:694-703)."""
    assert out.dtype == np.float32 and out.flags.c_contiguous
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    rank, in_dim = A.shape
    out_dim, S = out.shape
    tmp = np.zeros((rank, S), np.float32)
    lib().or_lora_addmm(_f(out), _f(A), _f(B), _f(x), _f(tmp), out_dim, rank, in_dim, S)


def cross_entropy(logits_tm: np.ndarray, targets: np.ndarray) -> float:
    """Mean CE of token-major logits [S, V] (cross_entropy_loss, training/cpu_ops.h:108-133)."""
    logits_tm = np.ascontiguousarray(logits_tm, np.float32)
    t = np.ascontiguousarray(targets, np.uint16)
    S, V = logits_tm.shape
    return float(lib().or_cross_entropy(_f(logits_tm), _u16(t), V, S))


def rope_tables(seq: int, hd: int, theta: float):
    c = np.zeros((seq, hd // 2), np.float32)
    s = np.zeros((seq, hd // 2), np.float32)
    lib().or_rope_tables(_f(c), _f(s), seq, hd, np.float32(theta))
    return c, s


# ---------------- model ----------------
@dataclass
class ModelCfg:
    dim: int
    hidden: int
    heads: int
    kv_heads: int
    hd: int
    seq: int
    nlayers: int
    vocab: int
    rank: int = 8
    rope_theta: float = 100000.0
    res_alpha: float = 1.0
    lora_ffn: bool = False  # --lora-ffn: adapters on W1, W2, W3 too

    @property
    def q_dim(self):
        return self.heads * self.hd

    @property
    def kv_dim(self):
        return self.kv_heads * self.hd


class OracleModel:
    """Reference-layout fp32 weights wired into the C oracle."""

    def __init__(self, cfg: ModelCfg, weights: dict, embed: np.ndarray, cembed: np.ndarray):
        self.cfg = cfg
        self.w = weights  # name -> list of [out, in] float32 arrays
        self.embed = np.ascontiguousarray(embed, np.float32)
        self.cembed = np.ascontiguousarray(cembed, np.float32)
        self._keep = []
        m = _Model()
        for f in ("dim", "hidden", "heads", "kv_heads", "hd", "seq", "nlayers", "vocab", "rank"):
            setattr(m, f, getattr(cfg, f))
        m.cv = self.cembed.shape[0]
        m.lora_ffn = int(getattr(cfg, "lora_ffn", False))
        m.rope_theta = cfg.rope_theta
        m.res_alpha = cfg.res_alpha
        for n in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"):
            arrs = [np.ascontiguousarray(a, np.float32) for a in weights[n]]
            self._keep.append(arrs)
            ptrs = (C.POINTER(C.c_float) * cfg.nlayers)(*[_f(a) for a in arrs])
            self._keep.append(ptrs)
            setattr(m, n, ptrs)
        m.embed = _f(self.embed)
        m.cembed = _f(self.cembed)
        self.m = m

    def forward_loss(self, theta: np.ndarray, tokens: np.ndarray, ctargets: np.ndarray, taps: dict | None = None):
        tokens = np.ascontiguousarray(tokens, np.uint16)
        ctargets = np.ascontiguousarray(ctargets, np.uint16)
        t = None
        if taps is not None:
            t = _Taps()
            for k, v in taps.items():
                setattr(t, k, _f(v))
        return float(lib().or_forward_loss(C.byref(self.m), _f(theta), _u16(tokens), _u16(ctargets),
                                           C.byref(t) if t is not None else None))

    def p16_grad(self, theta: np.ndarray, tokens, ctargets):
        """(loss, gradient in theta layout) of one sequence (backprop-LoRA, P16)."""
        grad = np.zeros_like(theta)
        loss = lib().or_p16_grad(C.byref(self.m), _f(np.ascontiguousarray(theta, np.float32)),
                                 _u16(np.ascontiguousarray(tokens, np.uint16)),
                                 _u16(np.ascontiguousarray(ctargets, np.uint16)), _f(grad))
        return float(loss), grad

    def full_grad(self, theta: np.ndarray, tokens, ctargets, c2f=None):
        """(loss, theta-layout grad, dW per layer (dict name -> list), embedding grad) of one sequence."""
        cfg = self.cfg
        D, H, QD, KVD = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim
        shapes = [("Wq", (QD, D)), ("Wk", (KVD, D)), ("Wv", (KVD, D)), ("Wo", (D, QD)), ("W1", (H, D)),
                  ("W2", (D, H)), ("W3", (H, D))]
        per_l = sum(a * b for _, (a, b) in shapes)
        dw = np.zeros(per_l * cfg.nlayers, np.float32)
        gembed = np.zeros((cfg.vocab, D), np.float32)
        grad = np.zeros_like(theta)
        cp = None
        if c2f is not None:
            c2f = np.ascontiguousarray(c2f, np.int32)
            cp = c2f.ctypes.data_as(C.POINTER(C.c_int32))
        loss = lib().or_full_grad(C.byref(self.m), _f(np.ascontiguousarray(theta, np.float32)),
                                  _u16(np.ascontiguousarray(tokens, np.uint16)),
                                  _u16(np.ascontiguousarray(ctargets, np.uint16)), _f(grad), _f(dw), _f(gembed), cp)
        out = {n: [] for n, _ in shapes}
        o = 0
        for l in range(cfg.nlayers):
            for n, (a, b) in shapes:
                out[n].append(dw[o:o + a * b].reshape(a, b))
                o += a * b
        return float(loss), grad, out, gembed

    def mezo_step(self, theta: np.ndarray, tokens, ctargets, seed: int, eps: float, lr: float):
        lp, lm, g = C.c_float(), C.c_float(), C.c_float()
        lib().or_mezo_step(C.byref(self.m), _f(theta), _u16(np.ascontiguousarray(tokens, np.uint16)),
                           _u16(np.ascontiguousarray(ctargets, np.uint16)), seed, np.float32(eps), np.float32(lr),
                           C.byref(lp), C.byref(lm), C.byref(g))
        return lp.value, lm.value, g.value


def adam(w: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray, t: int, lr: float, b1: float = 0.9,
         b2: float = 0.95, eps: float = 1e-8, wd: float = 0.0) -> None:
    """adam_update (training/cpu_ops.h:62-104) in place on w, m, v."""
    for a in (w, g, m, v):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    lib().or_adam(_f(w), _f(g), _f(m), _f(v), w.size, t, np.float32(lr), np.float32(b1), np.float32(b2),
                  np.float32(eps), np.float32(wd))


# ---------------- reference-compiled library ----------------
def ref_lib(model: str):
    """oracle/_ref/libref_<model>.so, or None when it was not built (no reference tree)."""
    p = HERE / "_ref" / f"libref_{model}.so"
    if not p.exists():
        return None
    L = C.CDLL(str(p))
    L.ref_cross_entropy.restype = C.c_float
    L.ref_forward_loss.restype = C.c_float
    L.ref_forward_loss_ffn.restype = C.c_float
    L.ref_p16_grad.restype = C.c_float
    L.ref_p16_grad_dw.restype = C.c_float
    return L
