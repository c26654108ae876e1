"""Checkpoint files of the reference, restated in numpy. TEST INFRASTRUCTURE ONLY:
the library never imports this module; tests use it to check the files that
libb2p.so writes and to make files for it to read.

BLZT v4 (little-endian):
  * header: CkptHdr, training/config.h:99-108 — 10 int32, 2 float32, 3 float64,
    6 int32 = 96 bytes (the format string of generate.py:55);
  * per layer (train.m:189-203, train_mezo.m:718-740): Wq Wk Wv Wo W1 W2 W3
    rms_att rms_ffn, then the Adam pairs Wq.m Wq.v Wk.m Wk.v ... rms_ffn.m rms_ffn.v;
  * rms_final, its m, v; embed [vocab, dim], its m, v (train.m:204-207).
LORA sidecar (lora_save_checkpoint, train_mezo.m:791-815): int32 magic
0x4C4F5241, rank, nlayers, adam_t; per layer Aq Bq Ak Bk Av Bv Ao Bo.

Pinned against the reference's own reader: tests/golden/make_ckpt_golden.py
writes a file with `write_blzt`, reads it back with generate.py's
load_checkpoint and records the file's SHA-256.
"""
from __future__ import annotations

import struct

import numpy as np

HDR_FMT = "<10i2f3d6i"
HDR_FIELDS = ("magic", "version", "step", "total_steps", "n_layers", "vocab_size", "dim", "hidden_dim", "n_heads",
              "seq_len", "lr", "loss", "cum_compile", "cum_train", "cum_wall", "cum_steps", "cum_batches", "adam_t",
              "kv_heads", "head_dim", "q_dim")
BLZT_MAGIC, LORA_MAGIC = 0x424C5A54, 0x4C4F5241
WEIGHTS = ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")
ADAPTERS = ("Aq", "Bq", "Ak", "Bk", "Av", "Bv", "Ao", "Bo")
assert struct.calcsize(HDR_FMT) == 96


def header(cfg, **kw) -> dict:
    """CkptHdr with the structural fields of `cfg` (oracle.ModelCfg) and the given scalars."""
    h = dict.fromkeys(HDR_FIELDS, 0)
    h.update(magic=BLZT_MAGIC, version=4, n_layers=cfg.nlayers, vocab_size=cfg.vocab, dim=cfg.dim,
             hidden_dim=cfg.hidden, n_heads=cfg.heads, seq_len=cfg.seq, kv_heads=cfg.kv_heads, head_dim=cfg.hd,
             q_dim=cfg.heads * cfg.hd)
    h.update(kw)
    return h


def pack_header(h: dict) -> bytes:
    return struct.pack(HDR_FMT, *[h[k] for k in HDR_FIELDS])


def unpack_header(b: bytes) -> dict:
    return dict(zip(HDR_FIELDS, struct.unpack(HDR_FMT, b[:96])))


def _f32(a) -> bytes:
    return np.ascontiguousarray(a, np.float32).tobytes()


def write_blzt(path, h: dict, layers: list, rms_final, embed, adam: dict | None = None):
    """layers[l]: dict with WEIGHTS + rms_att, rms_ffn. adam (None = zero slots, the MeZO
    writer): {'layers': [ {name: (m, v)} ], 'rms_final': (m, v), 'embed': (m, v)}."""
    with open(path, "wb") as f:
        f.write(pack_header(h))
        for l, lw in enumerate(layers):
            names = WEIGHTS + ("rms_att", "rms_ffn")
            for k in names:
                f.write(_f32(lw[k]))
            for k in names:
                if adam is None:
                    z = np.zeros(np.size(lw[k]), np.float32)
                    f.write(_f32(z) + _f32(z))
                else:
                    m, v = adam["layers"][l][k]
                    f.write(_f32(m) + _f32(v))
        f.write(_f32(rms_final))
        zf = np.zeros(np.size(rms_final), np.float32)
        f.write(_f32(zf) * 2 if adam is None else _f32(adam["rms_final"][0]) + _f32(adam["rms_final"][1]))
        f.write(_f32(embed))
        ze = np.zeros(np.size(embed), np.float32)
        f.write(_f32(ze) * 2 if adam is None else _f32(adam["embed"][0]) + _f32(adam["embed"][1]))


def read_blzt(path, cfg) -> dict:
    """Everything in a BLZT v4 file (weights and Adam slots) for the shapes of `cfg`."""
    D, H, QD, KVD, V = cfg.dim, cfg.hidden, cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd, cfg.vocab
    shapes = {"Wq": (QD, D), "Wk": (KVD, D), "Wv": (KVD, D), "Wo": (D, QD), "W1": (H, D), "W2": (D, H),
              "W3": (H, D), "rms_att": (D,), "rms_ffn": (D,)}
    data = open(path, "rb").read()
    h = unpack_header(data)
    o = 96

    def take(shape):
        nonlocal o
        n = int(np.prod(shape))
        a = np.frombuffer(data, np.float32, n, o).reshape(shape).copy()
        o += 4 * n
        return a

    layers, adam = [], []
    for _ in range(cfg.nlayers):
        layers.append({k: take(s) for k, s in shapes.items()})
        adam.append({k: (take(s), take(s)) for k, s in shapes.items()})
    rms_final = take((D,))
    rf_adam = (take((D,)), take((D,)))
    embed = take((V, D))
    e_adam = (take((V, D)), take((V, D)))
    assert o == len(data), (o, len(data))
    return {"header": h, "layers": layers, "rms_final": rms_final, "embed": embed,
            "adam": {"layers": adam, "rms_final": rf_adam, "embed": e_adam}}


def write_lora(path, rank: int, adam_t: int, adapters: list):
    """adapters[l]: dict with ADAPTERS (fp32 arrays)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<4i", LORA_MAGIC, rank, len(adapters), adam_t))
        for ad in adapters:
            for k in ADAPTERS:
                f.write(_f32(ad[k]))


def read_lora(path, cfg) -> tuple[int, list]:
    D, QD, KVD, r = cfg.dim, cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd, cfg.rank
    shapes = {"Aq": (r, D), "Bq": (QD, r), "Ak": (r, D), "Bk": (KVD, r), "Av": (r, D), "Bv": (KVD, r),
              "Ao": (r, QD), "Bo": (D, r)}
    data = open(path, "rb").read()
    magic, rank, nl, adam_t = struct.unpack("<4i", data[:16])
    assert magic == LORA_MAGIC and rank == r and nl == cfg.nlayers
    o, out = 16, []
    for _ in range(nl):
        ad = {}
        for k, s in shapes.items():
            n = int(np.prod(s))
            ad[k] = np.frombuffer(data, np.float32, n, o).reshape(s).copy()
            o += 4 * n
        out.append(ad)
    assert o == len(data)
    return adam_t, out


def add_ba(W, B, A, sign: float):
    """W ± B·A in fp32 (lora_merge_weight, training/config.h:278-283, and the un-merge of
    train_mezo.m:1140-1149): the product summed over k in ascending order, then added to W."""
    acc = np.zeros(W.shape, np.float32)
    for k in range(A.shape[0]):
        acc = acc + B[:, k:k + 1].astype(np.float32) * A[k:k + 1, :].astype(np.float32)
    return (W + acc if sign > 0 else W - acc).astype(np.float32)


def adapters_of(theta, layout, cfg) -> list:
    """Per-layer adapters out of the flat trainable vector (perturbation order)."""
    D, QD, KVD, r = cfg.dim, cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd, cfg.rank
    shapes = {"Aq": (r, D), "Bq": (QD, r), "Ak": (r, D), "Bk": (KVD, r), "Av": (r, D), "Bv": (KVD, r),
              "Ao": (r, QD), "Bo": (D, r)}
    out = []
    for l in range(cfg.nlayers):
        b = l * layout.layer_size
        out.append({k: theta[b + getattr(layout, k): b + getattr(layout, k) + int(np.prod(s))].reshape(s)
                    for k, s in shapes.items()})
    return out


def merged(layers: list, adapters: list, sign: float) -> list:
    """Copy of `layers` with Wq/Wk/Wv/Wo ± B·A of each layer's adapters."""
    out = []
    for lw, ad in zip(layers, adapters):
        n = dict(lw)
        for w, a, b in (("Wq", "Aq", "Bq"), ("Wk", "Ak", "Bk"), ("Wv", "Av", "Bv"), ("Wo", "Ao", "Bo")):
            n[w] = add_ba(np.asarray(lw[w], np.float32), ad[b], ad[a], sign)
        out.append(n)
    return out
