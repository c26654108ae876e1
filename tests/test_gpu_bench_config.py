"""The benchmarked MeZO configuration itself against the oracle.

bench.py's headline step evaluates, per GPU, 8 SmolLM2-360M sequences of 256
tokens under 4 seeds x (+eps, -eps): 64 groups, 16,384 token rows in one
batched forward, with the CTA-pair projection engine, the tcgen05 attention
kernel (persistent, work counter over 64 sequences x 5 KV heads x 2 query
blocks), per-variant LoRA-down operands for 8 variants and programmatic
dependent launch, all at their defaults. The inputs here are bench.py's own
synthetic weights, LoRA init and token positions.

Gates (fp16 compute, fp32 accumulation):
  * every one of the 64 group losses equals the same (sequence, variant)
    evaluated alone on a model built for 2 groups, to 1e-5 nats;
  * for 2 of the 4 seeds, both signs over all 8 sequences (32 groups), each
    group loss is within 1e-3 nats of the oracle's forward (training/
    train_mezo.m:1528-1699 restated in oracle/oracle.c) at the same perturbed
    parameters, i.e. the per-step loss gate of the workload definition;
  * the loss pairs b2p_mezo_eval returns are the means of their 8 groups.
"""
import os

import numpy as np
import pytest

import bench
from autoane_b200.model import Config, Model
from oracle import oracle as O
from tests import _models as M

pytestmark = pytest.mark.gpu

EPS = np.float32(1e-3)


@pytest.fixture(scope="module")
def bench_setup(b2p):
    ws = [bench.synth_weights(l) for l in range(bench.DIMS["nlayers"])]
    weights = {k: [w[i] for w in ws] for i, k in enumerate(("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"))}
    embed = bench.synth_embed()
    theta = bench.synth_theta(bench.lora_layout())
    tokens = bench.token_stream()
    inp, tgt = bench.step_batch(tokens, 3, 0, bench.SEQS_PER_GPU)
    seeds = bench.step_seeds(3, 1)
    dims = {k: bench.DIMS[k] for k in ("dim", "hidden", "heads", "kv_heads", "head_dim", "seq", "nlayers", "vocab",
                                       "rank", "rope_theta")}
    models = []
    for groups in (2 * bench.SEEDS_PER_GPU * bench.SEQS_PER_GPU, 2):
        m = Model(Config(max_groups=groups, **dims))
        for l in range(bench.DIMS["nlayers"]):
            m.set_layer(l, *ws[l])
        m.set_embedding(embed, np.arange(bench.N_ACTIVE, dtype=np.int32))
        m.set_trainable(theta)
        models.append(m)
    yield weights, embed, theta, inp, tgt, seeds, models
    for m in models:
        m.close()


def test_bench_batch_groups_match_single_group_evaluations(bench_setup):
    weights, embed, theta, inp, tgt, seeds, (big, small) = bench_setup
    nseq, nseed = bench.SEQS_PER_GPU, bench.SEEDS_PER_GPU
    assert big.cfg.max_groups == 64 and inp.shape == (nseq, 256)
    pairs = big.mezo_eval(inp, tgt, seeds, float(EPS))
    groups = big.group_losses(2 * nseed * nseq)
    for v in range(2 * nseed):
        assert abs(pairs[v] - np.mean(groups[v * nseq:(v + 1) * nseq], dtype=np.float64)) < 1e-5
    worst = 0.0
    for v in range(2 * nseed):
        s = int(seeds[v // 2])
        var = (s, 1, EPS, 0.0) if v % 2 == 0 else (s, 2, EPS, np.float32(-2.0) * EPS)
        for q in range(nseq):
            alone = small.eval(inp[q], tgt[q], [var])[0]
            worst = max(worst, abs(float(groups[v * nseq + q]) - float(alone)))
    print(f"bench batch vs single-group evaluations: worst |dL| = {worst:.3e}")
    assert worst < 1e-5, worst


def test_bench_batch_groups_match_oracle(bench_setup):
    weights, embed, theta, inp, tgt, seeds, (big, _) = bench_setup
    nseq = bench.SEQS_PER_GPU
    cfg = M.SMOLLM2
    O.set_threads(os.cpu_count() or 1)
    cembed = np.ascontiguousarray(embed[:bench.N_ACTIVE])
    om = O.OracleModel(cfg, weights, embed, cembed)
    big.mezo_eval(inp, tgt, seeds, float(EPS))
    groups = big.group_losses(2 * bench.SEEDS_PER_GPU * nseq)
    worst = 0.0
    for si in (0, 3):  # first and last seed of the step: variants 2si (+eps) and 2si+1 (-eps)
        s = int(seeds[si])
        for sign, scales in ((0, [EPS]), (1, [EPS, np.float32(-2.0) * EPS])):
            th = theta.copy()
            for sc in scales:
                O.perturb_lora(th, cfg.nlayers, cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.rank, s, sc)
            v = 2 * si + sign
            for q in range(nseq):
                ref = om.forward_loss(th, inp[q], tgt[q])
                d = abs(float(groups[v * nseq + q]) - ref)
                worst = max(worst, d)
                assert d < 1e-3, (si, sign, q, float(groups[v * nseq + q]), ref)
    print(f"bench batch vs oracle (32 groups): worst |dL| = {worst:.3e}")
