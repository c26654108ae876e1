"""Data-parallel host logic on CPU: two gloo ranks drive oracle replicas through
autoane_b200.dp.DPMeZO; both must end bit-identical and equal to one process
applying the same seed-ordered update with every rank's loss pairs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from autoane_b200.dp import DPMeZO, step_seeds
from oracle import oracle as O
from tests import _models as M

CFG = O.ModelCfg(dim=128, hidden=256, heads=2, kv_heads=1, hd=64, seq=32, nlayers=2, vocab=512, rank=4,
                 rope_theta=10000.0)
N_ACTIVE = 300


class OracleReplica:
    """Host replica of the MeZO-LoRA-split math on the oracle (test infrastructure)."""

    def __init__(self, seed=3):
        self.syn = M.make_model(CFG, N_ACTIVE, seed=seed, b_scale=0.01)
        self.om = O.OracleModel(CFG, self.syn.weights, self.syn.embed, self.syn.cembed)
        self.theta = self.syn.theta.copy()

    def _perturbed(self, seed, scales):
        t = self.theta.copy()
        for s in scales:
            O.perturb_lora(t, CFG.nlayers, CFG.dim, CFG.q_dim, CFG.kv_dim, CFG.rank, int(seed), s)
        return t

    def mezo_eval(self, tokens, ctargets, seeds, eps):
        eps = np.float32(eps)
        out = []
        for s in seeds:
            for scales in ([eps], [eps, np.float32(-2.0) * eps]):
                t = self._perturbed(s, scales)
                out.append(np.mean([self.om.forward_loss(t, tokens[i], ctargets[i]) for i in range(len(tokens))]))
        return np.array(out, np.float32)

    def mezo_update(self, seeds, pairs, eps, lr):
        eps, lr = np.float32(eps), np.float32(lr)
        n = np.float32(len(seeds))
        for k, s in enumerate(seeds):
            g = np.float32((pairs[2 * k] - pairs[2 * k + 1]) / (np.float32(2.0) * eps))
            c = np.float32(np.float32(-lr * g) / n)
            O.perturb_lora(self.theta, CFG.nlayers, CFG.dim, CFG.q_dim, CFG.kv_dim, CFG.rank, int(s), c)


def batch(rank, step):
    toks = M.make_tokens(4096, N_ACTIVE, seed=11)
    syn = M.make_model(CFG, N_ACTIVE, seed=3)
    span = len(toks) - CFG.seq - 2
    seqs = [M.sample_sequence(toks, CFG.seq, syn.full_to_compact, (100 + 997 * (step * 7 + rank * 3 + i)) % span)
            for i in range(2)]
    return np.stack([s[0] for s in seqs]), np.stack([s[1] for s in seqs])


def worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        rep = OracleReplica()
        dp = DPMeZO(rep, seeds_per_rank=2, eps=1e-3, lr=1e-3)
        allp = []
        for step in range(2):
            tok, tgt = batch(rank, step)
            allp.append(dp.step(step, tok, tgt))
        q.put((rank, rep.theta.copy(), allp))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(300)
def test_two_gloo_ranks_stay_identical_and_match_serial_update():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(2)], key=lambda x: x[0])
    for r, th, info in res:
        assert th is not None, f"rank {r} failed: {info}"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, th0, p0), (r1, th1, p1) = res
    assert np.array_equal(th0.view(np.uint32), th1.view(np.uint32))
    # serial replay: the gathered pairs are rank-major and the update is seed-ordered
    ref = OracleReplica()
    for step in range(2):
        seeds = step_seeds(step, 2, 2)
        pairs = np.concatenate([ref.mezo_eval(*batch(r, step), seeds[2 * r:2 * r + 2], 1e-3) for r in range(2)])
        assert np.array_equal(pairs, p0[step])
        ref.mezo_update(seeds, pairs, 1e-3, 1e-3)
    assert np.array_equal(ref.theta.view(np.uint32), th0.view(np.uint32))


class _ThetaModel:
    def __init__(self, theta):
        self.theta = theta

    def get_trainable(self):
        return self.theta


def checks_worker(rank, world, port, q, diverge):
    """bench.rank_checks on gloo ranks: rank 1 perturbs one parameter by one ulp when `diverge`."""
    import datetime
    import torch
    import torch.distributed as dist
    try:
        import bench
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        theta = np.linspace(-1, 1, 1001, dtype=np.float32)
        if diverge and rank == 1:
            theta[500] = np.nextafter(theta[500], np.float32(2))
        out = bench.rank_checks(_ThetaModel(theta), 100.0 + 10.0 * rank, 10, world, torch.device("cpu"))
        q.put((rank, out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.timeout(300)
@pytest.mark.parametrize("diverge", [False, True])
def test_bench_rank_checks_detect_diverged_replicas(diverge):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=checks_worker, args=(r, 2, port, q, diverge)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(2)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    for r, out in res:
        assert isinstance(out, dict), f"rank {r}: {out}"
        assert out["rank_ms_per_step"] == {"min": 10.0, "max": 11.0}
        assert out["theta_identical_across_ranks"] is (not diverge)
