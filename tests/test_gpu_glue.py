"""Variant operands of the persistent RMSNorm + LoRA-down kernels (autoane_b200/csrc/kernels.cu:
norm_down_kernel, lora_down_kernel) across many variant groups.

Each CTA of those kernels walks a contiguous range of 16-row tiles and keeps the perturbed
operands of two variant groups in shared memory; a range that meets a third group restages a
slot at that group's first tile. 192 variants of one 128-token sequence give 24,576 rows: ranges
of 10-11 tiles over groups of 8 tiles, so most CTAs restage. A group's loss depends only on its
(sequence, variant), so evaluating a permutation of the variant list must permute the per-group
losses bit for bit; an operand slot read for the wrong group would make a loss follow the
group's position in the batch instead.
"""
import numpy as np
import pytest

from autoane_b200.model import Config, Model, load_synthetic
from tests import _models as M

pytestmark = pytest.mark.gpu


def test_restaged_variant_operands_follow_their_groups(b2p):
    cfg = M.small_cfg(nlayers=1, seq=128)
    nv = 192
    syn = M.make_model(cfg, n_active=3000, seed=11, b_scale=0.02, rms_jitter=0.05)
    model = Model(Config(dim=cfg.dim, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.hd,
                         seq=cfg.seq, nlayers=cfg.nlayers, vocab=cfg.vocab, rank=cfg.rank, rope_theta=cfg.rope_theta,
                         res_alpha=cfg.res_alpha, max_groups=nv))
    load_synthetic(model, syn.weights, syn.embed, syn.compact_to_full, syn.theta)
    toks = M.make_tokens(1 << 15, 3000, seed=11)
    inp, tgt = M.sample_sequence(toks, cfg.seq, syn.full_to_compact, 4242)
    # 8 seeds x 24 scales: every (seed, scale) pair distinct, so every group's operands differ
    variants = [(1000 + v % 8, 1, 1e-3 * (1 + v // 8), 0.0) for v in range(nv)]
    perm = np.random.default_rng(3).permutation(nv)
    model.eval(inp[None], tgt[None], variants)
    g1 = model.group_losses(nv)
    model.eval(inp[None], tgt[None], [variants[p] for p in perm])
    g2 = model.group_losses(nv)
    model.close()
    assert np.all(np.isfinite(g1))
    assert len(np.unique(g1)) > nv // 2, "variants should give distinct losses"
    bad = np.flatnonzero(g2 != g1[perm])
    assert bad.size == 0, f"{bad.size} groups changed with their position, first {bad[:8]}"
