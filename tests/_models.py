"""Seeded synthetic models and token streams shared by the tests.

Weights follow the workload definition: base projections N(0, 0.02²), RMS
weights 1 (optionally jittered), LoRA A ~ N(0, 1/r) and B = 0 (or small random
B so the LoRA-up path is exercised), tied embedding N(0, 0.02²). Token ids are
uniform over [0, n_active) so vocabulary compaction (cpu_ops.h:142-176) yields
a compact vocabulary of n_active ids.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from oracle import oracle as O


@dataclass
class Synth:
    cfg: O.ModelCfg
    weights: dict
    embed: np.ndarray
    cembed: np.ndarray
    compact_to_full: np.ndarray
    full_to_compact: np.ndarray
    theta: np.ndarray
    layout: object
    extra: dict = field(default_factory=dict)


def make_model(cfg: O.ModelCfg, n_active: int, seed: int = 42, b_scale: float = 0.0, rms_jitter: float = 0.0,
               w_std: float = 0.02) -> Synth:
    rng = np.random.default_rng(seed)
    L, D, H, QD, KVD, r = cfg.nlayers, cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.rank
    shapes = {"Wq": (QD, D), "Wk": (KVD, D), "Wv": (KVD, D), "Wo": (D, QD), "W1": (H, D), "W2": (D, H),
              "W3": (H, D)}
    weights = {k: [(rng.standard_normal(s, dtype=np.float32) * w_std).astype(np.float32) for _ in range(L)]
               for k, s in shapes.items()}
    embed = (rng.standard_normal((cfg.vocab, D), dtype=np.float32) * 0.02).astype(np.float32)
    # vocabulary compaction over ids [0, n_active): compact id == full id here
    full_to_compact = np.full(cfg.vocab, -1, np.int32)
    full_to_compact[:n_active] = np.arange(n_active)
    compact_to_full = np.arange(n_active, dtype=np.int32)
    cembed = np.ascontiguousarray(embed[compact_to_full])
    ffn = bool(getattr(cfg, "lora_ffn", False))
    lay = O.lora_layout_ffn(L, D, QD, KVD, H, r, ffn)
    theta = np.zeros(lay.total, np.float32)
    a_std = 1.0 / np.sqrt(r)
    for l in range(L):
        base = l * lay.layer_size
        for off, n in ((lay.Aq, r * D), (lay.Ak, r * D), (lay.Av, r * D), (lay.Ao, r * QD)):
            theta[base + off: base + off + n] = rng.standard_normal(n, dtype=np.float32) * a_std
        if b_scale:
            for off, n in ((lay.Bq, QD * r), (lay.Bk, KVD * r), (lay.Bv, KVD * r), (lay.Bo, D * r)):
                theta[base + off: base + off + n] = rng.standard_normal(n, dtype=np.float32) * b_scale
        if ffn:  # --lora-ffn adapters (train_mezo.m:1079-1091): A random, B small random when b_scale
            for off, n in ((lay.A1, r * D), (lay.A2, r * H), (lay.A3, r * D)):
                theta[base + off: base + off + n] = rng.standard_normal(n, dtype=np.float32) * a_std
            if b_scale:
                for off, n in ((lay.B1, H * r), (lay.B2, D * r), (lay.B3, H * r)):
                    theta[base + off: base + off + n] = rng.standard_normal(n, dtype=np.float32) * b_scale
        theta[base + lay.rms_att: base + lay.rms_att + D] = 1.0
        theta[base + lay.rms_ffn: base + lay.rms_ffn + D] = 1.0
        if rms_jitter:
            theta[base + lay.rms_att: base + lay.rms_ffn + D] += (
                rng.standard_normal(2 * D, dtype=np.float32) * rms_jitter)
    theta[lay.rms_final: lay.rms_final + D] = 1.0
    return Synth(cfg, weights, embed, cembed, compact_to_full, full_to_compact, theta.astype(np.float32), lay)


def make_tokens(n_tokens: int, n_active: int, seed: int = 42) -> np.ndarray:
    return np.random.default_rng(seed + 1).integers(0, n_active, n_tokens).astype(np.uint16)


def sample_sequence(tokens: np.ndarray, seq: int, full_to_compact: np.ndarray, pos: int):
    """input tokens and compact targets at `pos` (train_mezo.m:1946-1953)."""
    inp = tokens[pos: pos + seq].astype(np.uint16)
    tgt = full_to_compact[tokens[pos + 1: pos + 1 + seq]].astype(np.uint16)
    return inp, tgt


SMOLLM2 = O.ModelCfg(dim=960, hidden=2560, heads=15, kv_heads=5, hd=64, seq=256, nlayers=32, vocab=49152, rank=8,
                     rope_theta=100000.0)
AUTORESEARCH_MHA = O.ModelCfg(dim=512, hidden=1152, heads=8, kv_heads=8, hd=64, seq=128, nlayers=4, vocab=49152,
                              rank=8, rope_theta=10000.0)
AUTORESEARCH = O.ModelCfg(dim=512, hidden=1408, heads=8, kv_heads=2, hd=64, seq=128, nlayers=4, vocab=49152, rank=8,
                          rope_theta=10000.0)


def small_cfg(nlayers=2, seq=128, rank=8):
    """A SmolLM2-shaped (GQA 15/5, hd 64) slice with fewer layers, for fast parity runs."""
    return O.ModelCfg(dim=960, hidden=2560, heads=15, kv_heads=5, hd=64, seq=seq, nlayers=nlayers, vocab=49152,
                      rank=rank, rope_theta=100000.0)


def rms_slices(syn):
    """Slices of the RMS weights (rms_att, rms_ffn per layer, rms_final) in the trainable layout."""
    lay, D = syn.layout, syn.cfg.dim
    out = []
    for l in range(syn.cfg.nlayers):
        b = l * lay.layer_size
        out += [slice(b + lay.rms_att, b + lay.rms_att + D), slice(b + lay.rms_ffn, b + lay.rms_ffn + D)]
    out.append(slice(lay.rms_final, lay.rms_final + D))
    return out


CKPT_TINY = O.ModelCfg(dim=128, hidden=256, heads=2, kv_heads=1, hd=64, seq=64, nlayers=2, vocab=300, rank=8)


def ckpt_case(cfg, seed: int = 5):
    """Seeded checkpoint contents for `cfg`: per-layer frozen weights (fp16-representable, so a
    16-bit device copy widens back to the same fp32), RMS vectors, rms_final, embedding, adapters
    and the flat trainable vector holding the adapters and RMS vectors."""
    rng = np.random.default_rng(seed)
    D, H, QD, KVD, r = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.rank
    shapes = {"Wq": (QD, D), "Wk": (KVD, D), "Wv": (KVD, D), "Wo": (D, QD), "W1": (H, D), "W2": (D, H),
              "W3": (H, D)}
    lay = O.lora_layout(cfg.nlayers, D, QD, KVD, r)
    theta = np.zeros(lay.total, np.float32)
    layers = []
    for l in range(cfg.nlayers):
        lw = {k: (rng.standard_normal(s) * 0.02).astype(np.float16).astype(np.float32) for k, s in shapes.items()}
        b = l * lay.layer_size
        for k, s in (("Aq", (r, D)), ("Bq", (QD, r)), ("Ak", (r, D)), ("Bk", (KVD, r)), ("Av", (r, D)),
                     ("Bv", (KVD, r)), ("Ao", (r, QD)), ("Bo", (D, r))):
            n = s[0] * s[1]
            scale = 1.0 / np.sqrt(r) if k[0] == "A" else 0.01
            theta[b + getattr(lay, k): b + getattr(lay, k) + n] = rng.standard_normal(n) * scale
        for k in ("rms_att", "rms_ffn"):
            v = (1.0 + 0.05 * rng.standard_normal(D)).astype(np.float32)
            theta[b + getattr(lay, k): b + getattr(lay, k) + D] = v
            lw[k] = v
        layers.append(lw)
    rms_final = (1.0 + 0.05 * rng.standard_normal(D)).astype(np.float32)
    theta[lay.rms_final: lay.rms_final + D] = rms_final
    embed = (rng.standard_normal((cfg.vocab, D)) * 0.02).astype(np.float32)
    return layers, rms_final, embed, theta, lay
