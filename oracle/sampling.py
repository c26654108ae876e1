"""The reference host loop's integer and index work, restated. TEST INFRASTRUCTURE ONLY:
the library and the host loop never import this module; tests use it to check them.

  * drand48 / srand48: the POSIX 48-bit linear congruential generator the reference
    calls from libc (X <- (0x5DEECE66D * X + 0xB) mod 2^48; srand48(s) sets the high
    32 bits of X to the low 32 bits of s and the low 16 bits to 0x330E; drand48()
    returns X / 2^48). Pinned against the host libc in tests/test_host_loop.py.
  * training positions: srand48(seed + step * 7919); pos = (size_t)(drand48() *
    (train_tokens - SEQ - 1)) with train_tokens = (size_t)(n_tokens * 0.9)
    (training/train_mezo.m:1240, 1946-1949);
  * validation positions: srand48(999), then val_start + (size_t)(drand48() *
    (val_tokens - SEQ - 1)) for 10 windows (train_mezo.m:3150-3158);
  * vocab_map_build (training/cpu_ops.h:142-166): used ids in ascending order;
  * LoRA init: srand48(seed + 12345), per layer A_q, A_k, A_v, A_o (and with
    --lora-ffn A_1, A_3, A_2) each a_scale * (2 * drand48() - 1) with a_scale =
    1/sqrtf(r), B = 0 (train_mezo.m:1056-1093);
  * MeZO cosine schedule (train_mezo.m:3133-3135).
"""
from __future__ import annotations

import math

import numpy as np

_A, _C, _M = 0x5DEECE66D, 0xB, (1 << 48) - 1


class Drand48:
    """srand48/drand48 (POSIX)."""

    def __init__(self, seed: int):
        self.x = ((seed & 0xFFFFFFFF) << 16) | 0x330E

    def next(self) -> float:
        self.x = (_A * self.x + _C) & _M
        return self.x / float(1 << 48)

    def fill(self, n: int) -> np.ndarray:
        """n consecutive drand48() values as float64."""
        out = np.empty(n, np.float64)
        x = self.x
        for i in range(n):
            x = (_A * x + _C) & _M
            out[i] = x
        self.x = x
        return out / float(1 << 48)


def train_split(n_tokens: int) -> int:
    return int(np.float64(n_tokens) * 0.9)


def train_position(seed: int, step: int, n_tokens: int, seq: int) -> int:
    max_pos = train_split(n_tokens) - seq - 1
    return int(Drand48(seed + step * 7919).next() * float(max_pos))


def val_positions(n_tokens: int, seq: int, n: int = 10) -> list[int]:
    vs = train_split(n_tokens)
    g = Drand48(999)
    return [vs + int(g.next() * float(n_tokens - vs - seq - 1)) for _ in range(n)]


def vocab_map_build(tokens: np.ndarray, vocab: int):
    used = np.zeros(vocab, bool)
    used[tokens] = True
    c2f = np.nonzero(used)[0].astype(np.int32)
    f2c = np.full(vocab, -1, np.int32)
    f2c[c2f] = np.arange(len(c2f), dtype=np.int32)
    return f2c, c2f


def lora_init(theta: np.ndarray, layout, cfg, seed: int, ffn: bool = False) -> None:
    """Write the reference's LoRA A init into theta (B blocks zeroed) in place."""
    r, D, QD, H = cfg.rank, cfg.dim, cfg.q_dim, cfg.hidden
    a_scale = np.float64(np.float32(1.0) / np.sqrt(np.float32(r), dtype=np.float32))
    g = Drand48(seed + 12345)
    for l in range(cfg.nlayers):
        b = l * layout.layer_size
        blocks = [(layout.Aq, r * D), (layout.Ak, r * D), (layout.Av, r * D), (layout.Ao, r * QD)]
        if ffn:
            blocks += [(layout.A1, r * D), (layout.A3, r * D), (layout.A2, r * H)]
        for off, n in blocks:
            theta[b + off: b + off + n] = (a_scale * (2.0 * g.fill(n) - 1.0)).astype(np.float32)
        for off, n in ((layout.Bq, QD * r), (layout.Bk, cfg.kv_dim * r), (layout.Bv, cfg.kv_dim * r),
                       (layout.Bo, D * r)):
            theta[b + off: b + off + n] = 0.0


def mezo_lr(base_lr: float, step: int, start: int, total: int) -> np.float32:
    """lr after step `step` (train_mezo.m:3133-3135), float32 arithmetic as in C."""
    base = np.float32(base_lr)
    min_lr = np.float32(base * np.float32(0.1))
    decay = np.float32(np.float32(step - start) / np.float32(total - start))
    c = np.float32(math.cos(np.float32(math.pi * float(decay))))
    return np.float32(min_lr + np.float32(np.float32(0.5) * np.float32(np.float32(1.0) + c)) * np.float32(base - min_lr))
