"""Data-parallel MeZO-LoRA over ranks, one process per GPU.

Every rank holds a full replica (frozen base weights + the trainable LoRA/RMS
parameters). A step:
  1. the global seed list of the step is seeds[k] = step * 1000003 + base + k,
     k < world * seeds_per_rank (the reference's per-step seed,
     training/train_mezo.m:1956, extended to several directions per step);
  2. rank r evaluates its own seeds k in [r*S, (r+1)*S) at θ+εz and θ-εz over
     its own sequences (one batched forward);
  3. the per-seed loss pairs are all-gathered (world * S * 2 floats);
  4. every rank applies the same seed-ordered update θ += c_k z_k with
     c_k = -lr * g_k / (world * S), g_k = (L+_k - L-_k) / (2ε) — the averaged
     K-direction update of train_mezo.m:2751-2768 — so replicas stay bit-identical.

The replica is any object with
    mezo_eval(tokens, ctargets, seeds, eps) -> float32[2 * len(seeds)]
    mezo_update(seeds, loss_pairs, eps, lr) -> None
(autoane_b200.model.Model on a GPU). The exchange uses torch.distributed
(NCCL between GPUs; gloo works for host-only replicas).
"""
from __future__ import annotations

import numpy as np


def step_seeds(step: int, world: int, seeds_per_rank: int, base: int = 42) -> np.ndarray:
    """All seeds of a step, rank-major: rank r owns seeds[r*S:(r+1)*S]."""
    return np.array([step * 1000003 + base + k for k in range(world * seeds_per_rank)], np.uint64)


def local_seeds(seeds: np.ndarray, rank: int, seeds_per_rank: int) -> np.ndarray:
    return seeds[rank * seeds_per_rank:(rank + 1) * seeds_per_rank]


class DPMeZO:
    """Host-side driver of one data-parallel MeZO step over a process group."""

    def __init__(self, replica, seeds_per_rank: int = 4, eps: float = 1e-3, lr: float = 1e-4, group=None,
                 device=None, base_seed: int = 42):
        import torch.distributed as dist
        self.replica = replica
        self.S = seeds_per_rank
        self.eps = np.float32(eps)
        self.lr = np.float32(lr)
        self.group = group
        self.dist = dist
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device
        self.base = base_seed

    def step(self, step: int, tokens, ctargets) -> np.ndarray:
        """Evaluate this rank's seeds on its sequences, exchange, update. Returns all loss pairs."""
        import torch
        seeds = step_seeds(step, self.world, self.S, self.base)
        mine = local_seeds(seeds, self.rank, self.S)
        pairs = np.asarray(self.replica.mezo_eval(tokens, ctargets, mine, float(self.eps)), np.float32)
        if self.world > 1:
            t = torch.from_numpy(pairs.copy())
            if self.device is not None:
                t = t.to(self.device)
            out = torch.empty(self.world * pairs.size, dtype=torch.float32, device=t.device)
            self.dist.all_gather_into_tensor(out, t, group=self.group)
            gathered = out.cpu().numpy()
        else:
            gathered = pairs
        if not np.all(np.isfinite(gathered)):
            raise FloatingPointError(f"non-finite loss pair at step {step}: {gathered}")
        self.replica.mezo_update(seeds, np.ascontiguousarray(gathered, np.float32), float(self.eps), float(self.lr))
        return gathered
