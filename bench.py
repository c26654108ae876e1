#!/usr/bin/env python
"""MeZO-LoRA-split throughput on SmolLM2-360M shapes, data-parallel over N B200s.

Workload (one "step", every GPU): 8 independent synthetic 256-token sequences,
4 perturbation seeds of its own, each seed evaluated at θ+εz and θ-εz over all
8 sequences (64 sequence-forwards per GPU), the per-seed loss pairs all-gathered
over NCCL, then the same seed-ordered LoRA/RMS update on every replica.

Metric unit: one "seq-step" is one ±ε forward pair over one 256-token sequence,
i.e. the forward work of one reference MeZO-LoRA-split step (train_mezo.m:2938-3012);
a step of this workload performs 32 seq-steps per GPU. `value` is the whole-job
seq-step rate with inputs resident in HBM, timed with CUDA events on the model
stream; `e2e` is the same rate through the host-buffer C ABI (b2p_mezo_eval /
b2p_mezo_update), host->device copies and the loss read-back inside the region.

Run:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
(N > 1 under torch.distributed.run, one rank per GPU.)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DIMS = dict(dim=960, hidden=2560, heads=15, kv_heads=5, head_dim=64, seq=256, nlayers=32, vocab=49152, rank=8,
            rope_theta=100000.0)
N_ACTIVE = 16893          # compact vocabulary (ids 0..16892)
N_TOKENS = 20_000_000     # synthetic token stream
SEQS_PER_GPU = 8
SEEDS_PER_GPU = 4
EPS = np.float32(1e-3)
LR = np.float32(1e-4)
REF_STEPS_PER_S = 3.82    # reference best: ANE conv-fused MeZO-LoRA-split r8, M2 Pro (README.md:16)


def fwd_flops_per_seq(ffn: bool = False) -> float:
    """Algorithmic FLOPs of one 256-token forward (projections + lm-head + LoRA + dense attention)."""
    d = DIMS
    s, D, H, r = d["seq"], d["dim"], d["hidden"], d["rank"]
    qd, kvd = d["heads"] * d["head_dim"], d["kv_heads"] * d["head_dim"]
    proj = 2 * s * (D * (qd + 2 * kvd) + qd * D + 3 * D * H)
    lora = 2 * s * r * ((3 * D + qd) + (qd + 2 * kvd + D))  # LoRA-down (A·x) + LoRA-up (B·U)
    if ffn:  # --lora-ffn: A1, A3 over xn2, A2 over the gated activation; B1, B3, B2
        lora += 2 * s * r * ((2 * D + H) + (2 * H + D))
    attn = 2 * 2 * d["heads"] * s * s * d["head_dim"]
    head = 2 * s * N_ACTIVE * D
    return float(d["nlayers"] * (proj + lora + attn) + head)


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def synth_weights(layer: int):
    rng = np.random.default_rng([42, layer])
    D, H = DIMS["dim"], DIMS["hidden"]
    qd, kvd = DIMS["heads"] * DIMS["head_dim"], DIMS["kv_heads"] * DIMS["head_dim"]
    shapes = [(qd, D), (kvd, D), (kvd, D), (D, qd), (H, D), (D, H), (H, D)]
    return [rng.standard_normal(s, dtype=np.float32) * np.float32(0.02) for s in shapes]


def synth_embed():
    rng = np.random.default_rng([42, 10_000])
    return rng.standard_normal((DIMS["vocab"], DIMS["dim"]), dtype=np.float32) * np.float32(0.02)


def synth_theta(layout):
    """LoRA A ~ N(0, 1/r), B = 0, RMS weights 1 (workload definition)."""
    rng = np.random.default_rng([42, 20_000])
    L, D, r, H = DIMS["nlayers"], DIMS["dim"], DIMS["rank"], DIMS["hidden"]
    qd = DIMS["heads"] * DIMS["head_dim"]
    theta = np.zeros(layout["total"], np.float32)
    a_blocks = [("Aq", r * D), ("Ak", r * D), ("Av", r * D), ("Ao", r * qd)]
    if "A1" in layout:
        a_blocks += [("A1", r * D), ("A2", r * H), ("A3", r * D)]
    for l in range(L):
        b = l * layout["layer"]
        for name, n in a_blocks:
            off = layout[name]
            theta[b + off:b + off + n] = rng.standard_normal(n, dtype=np.float32) / np.float32(np.sqrt(r))
        theta[b + layout["rms_att"]:b + layout["rms_att"] + 2 * D] = 1.0
    theta[layout["rms_final"]:] = 1.0
    return theta


def lora_layout(ffn: bool = False):
    """Trainable layout in perturb_lora_weights order (train_mezo.m:566-587)."""
    D, r, H = DIMS["dim"], DIMS["rank"], DIMS["hidden"]
    qd, kvd = DIMS["heads"] * DIMS["head_dim"], DIMS["kv_heads"] * DIMS["head_dim"]
    o, lay = 0, {}
    blocks = [("Aq", r * D), ("Bq", qd * r), ("Ak", r * D), ("Bk", kvd * r), ("Av", r * D), ("Bv", kvd * r),
              ("Ao", r * qd), ("Bo", D * r)]
    if ffn:
        blocks += [("A1", r * D), ("B1", H * r), ("A2", r * H), ("B2", D * r), ("A3", r * D), ("B3", H * r)]
    for name, n in blocks + [("rms_att", D), ("rms_ffn", D)]:
        lay[name] = o
        o += n
    lay["layer"] = o
    lay["rms_final"] = DIMS["nlayers"] * o
    lay["total"] = lay["rms_final"] + D
    return lay


def token_stream():
    return np.random.default_rng([42, 30_000]).integers(0, N_ACTIVE, N_TOKENS, dtype=np.int64).astype(np.uint16)


def step_batch(tokens, step: int, rank: int, nseq: int):
    """nseq sequences at seeded positions of the training split (train_mezo.m:1946-1953 analogue)."""
    rng = np.random.default_rng([7919, step, rank])
    train = int(len(tokens) * 0.9)
    pos = rng.integers(0, train - DIMS["seq"] - 1, nseq)
    inp = np.stack([tokens[p:p + DIMS["seq"]] for p in pos])
    tgt = np.stack([tokens[p + 1:p + 1 + DIMS["seq"]] for p in pos])  # compact id == full id here
    return np.ascontiguousarray(inp), np.ascontiguousarray(tgt)


def step_seeds(step: int, world: int):
    return np.array([step * 1000003 + 42 + k for k in range(SEEDS_PER_GPU * world)], np.uint64)


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [v for v in sm if v > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# --------------------------------------------------------------------------- CPU reference / baseline
def host_cores():
    """(logical CPUs, physical cores) of this host."""
    try:
        import psutil
        phys = psutil.cpu_count(logical=False)
    except Exception:
        phys = None
    return os.cpu_count() or 1, phys


def cpu_reference_rate(max_seconds: float = 20.0, max_steps: int = 6, min_steps: int = 2, weights=None, embed=None,
                       threads: int | None = None):
    """MeZO-LoRA-split steps/s of the CPU reference path on this host's cores (one step = one seq-step).

    Uses the reference's own cpu_ops.h compiled from the AutoANE sources (oracle/_ref) for the
    forward when that library was built, otherwise the oracle restatement (oracle/liboracle.so).
    `threads` BLAS threads (default: every logical CPU)."""
    from oracle import oracle as O
    threads = threads or os.cpu_count() or 1
    O.set_threads(threads)
    cfg = O.ModelCfg(dim=DIMS["dim"], hidden=DIMS["hidden"], heads=DIMS["heads"], kv_heads=DIMS["kv_heads"],
                     hd=DIMS["head_dim"], seq=DIMS["seq"], nlayers=DIMS["nlayers"], vocab=DIMS["vocab"],
                     rank=DIMS["rank"], rope_theta=DIMS["rope_theta"])
    if weights is None:
        ws = [synth_weights(l) for l in range(DIMS["nlayers"])]
        weights = {k: [w[i] for w in ws] for i, k in enumerate(("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"))}
    if embed is None:
        embed = synth_embed()
    cembed = np.ascontiguousarray(embed[:N_ACTIVE])
    lay = lora_layout()
    theta = synth_theta(lay)
    tokens = token_stream()
    ref = O.ref_lib("smollm2_360m")
    kind = "reference" if ref is not None else "port"
    om = O.OracleModel(cfg, weights, embed, cembed)
    if ref is not None:
        step_fn = _ref_step_fn(ref, cfg, weights, embed, cembed, lay)
    else:
        def step_fn(th, inp, tgt, seed):
            om.mezo_step(th, inp, tgt, seed, float(EPS), float(LR))
    done, t0 = 0, time.perf_counter()
    while done < max_steps and (done < min_steps or time.perf_counter() - t0 < max_seconds):
        inp, tgt = step_batch(tokens, done, 0, 1)
        step_fn(theta, inp[0], tgt[0], int(done * 1000003 + 42))
        done += 1
    dt = time.perf_counter() - t0
    return {"value": done / dt, "unit": "seq-steps/s", "cores": threads, "kind": kind,
            "sample": f"{done} MeZO-LoRA-split steps (1 seed, 1x256-token sequence each, +eps/-eps forwards and "
                      f"update), SmolLM2-360M shapes, fp32, {threads} threads; "
                      + ("forward = reference training/cpu_ops.h compiled from source + transcribed DO_FORWARD_PASS"
                         if kind == "reference" else "forward = oracle restatement")}


def _ref_step_fn(ref, cfg, weights, embed, cembed, lay):
    """MeZO step body (train_mezo.m:2938-3012) over the reference-compiled forward (oracle/_ref)."""
    import ctypes as C
    from oracle import oracle as O
    F = C.POINTER(C.c_float)
    keep = []

    def f(a):
        return a.ctypes.data_as(F)

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p

    wp = [plist(weights[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")]
    ref.ref_forward_loss.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                          C.POINTER(C.c_uint16), C.POINTER(C.c_uint16)]

    def fwd(theta, inp, tgt):
        lora, rms = [], []
        for l in range(cfg.nlayers):
            b = l * lay["layer"]
            for k in ("Aq", "Bq", "Ak", "Bk", "Av", "Bv", "Ao", "Bo"):
                lora.append(theta[b + lay[k]:])
            rms += [theta[b + lay["rms_att"]:], theta[b + lay["rms_ffn"]:]]
        return ref.ref_forward_loss(*wp, plist(lora), plist(rms), f(theta[lay["rms_final"]:]), f(embed), f(cembed),
                                    cembed.shape[0], cfg.rank, C.c_float(cfg.res_alpha),
                                    inp.ctypes.data_as(C.POINTER(C.c_uint16)),
                                    tgt.ctypes.data_as(C.POINTER(C.c_uint16)))

    def step(theta, inp, tgt, seed):
        args = (cfg.nlayers, cfg.dim, cfg.q_dim, cfg.kv_dim, cfg.rank, seed)
        O.perturb_lora(theta, *args, EPS)
        lp = fwd(theta, inp, tgt)
        O.perturb_lora(theta, *args, np.float32(-2.0) * EPS)
        lm = fwd(theta, inp, tgt)
        O.perturb_lora(theta, *args, EPS)
        g = np.float32((np.float32(lp) - np.float32(lm)) / (np.float32(2.0) * EPS))
        O.perturb_lora(theta, *args, np.float32(-LR * g))

    return step


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    # Each timed step is one bounded CPU sample: a single reference MeZO step (one seq-step).
    # Steps beyond what fits in ~90 s of CPU time are not run; the rate is over the steps timed.
    r = cpu_reference_rate(max_seconds=90.0, max_steps=max(2, args.steps), min_steps=2)
    line = {"metric": "MeZO-LoRA steps/s SmolLM2-360M @1/2/4/8 B200; proj-GEMM % of TC peak", "impl": "reference",
            "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / r["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": r["value"] / REF_STEPS_PER_S, "dtype": "f32", "data": "synthetic",
            "config": workload_config(world) | {"sample": r["sample"]},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def rank_checks(model, dev_ms_local: float, steps: int, world: int, dev):
    """N > 1 only, called by every rank at the same point: each rank's device ms per step
    (the spread between ranks separates skew from the collective's own cost) and a
    bit-identity check of the trainable parameters across ranks (SHA-256 of θ)."""
    import hashlib

    import torch
    import torch.distributed as dist
    if world == 1:
        return None
    t = torch.tensor([dev_ms_local / steps], device=dev, dtype=torch.float64)
    allt = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(allt, t)
    digest = hashlib.sha256(model.get_trainable().tobytes()).digest()[:8]
    hv = torch.tensor([int.from_bytes(digest, "little", signed=True)], device=dev, dtype=torch.int64)
    allh = [torch.zeros_like(hv) for _ in range(world)]
    dist.all_gather(allh, hv)
    ms = [float(x.item()) for x in allt]
    return {"rank_ms_per_step": {"min": round(min(ms), 4), "max": round(max(ms), 4)},
            "theta_identical_across_ranks": len({int(x.item()) for x in allh}) == 1}


def workload_config(world: int, ffn: bool = False):
    adapters = "adapters on Wq/Wk/Wv/Wo/W1/W2/W3 (--lora-ffn)" if ffn else "adapters on Wq/Wk/Wv/Wo"
    return {"workload": "DP MeZO-LoRA-split r8, SmolLM2-360M shapes (32L, d960, 15/5 heads, FFN 2560, "
                        f"compact vocab 16893), SEQ 256; {adapters}; per GPU 8 sequences x 4 seeds x (+eps, -eps)",
            "model": "SmolLM2-360M-shaped (random init)", "global_batch": SEQS_PER_GPU * world, "seq_len": DIMS["seq"],
            "parallelism": f"dp{world}", "seeds_per_gpu": SEEDS_PER_GPU, "lora_rank": DIMS["rank"],
            "eps": float(EPS), "lr": float(LR), "seq_steps_per_step": SEQS_PER_GPU * SEEDS_PER_GPU * world,
            "l2": "inputs larger than L2 (661 MB of 16-bit weights streamed per step)",
            "vs_baseline_ref": f"{REF_STEPS_PER_S} steps/s, M2 Pro ANE conv-fused (README.md:16)"}


# --------------------------------------------------------------------------- B200 arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--dtype", choices=["f16", "bf16"], default="f16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-profile", action="store_true", help="skip the in-region per-GEMM CUDA events")
    ap.add_argument("--lora-ffn", action="store_true", help="MeZO workload with LoRA on W1/W2/W3 too")
    ap.add_argument("--p16-seqs", type=int, default=P16_SEQS_PER_GPU, help="sequences per GPU per P16 step")
    ap.add_argument("--full-seqs", type=int, default=32, help="sequences per GPU per full-backprop step")
    ap.add_argument("--workload", choices=["mezo", "p16", "full", "gemm"], default="mezo",
                    help="mezo: the headline DP MeZO-LoRA-split step; p16: DP backprop-LoRA step; "
                         "gemm: projection-GEMM sweep (one line per shape)")
    args = ap.parse_args()
    if args.workload == "gemm":
        return run_gemm_sweep(args)
    if args.impl == "reference":
        return run_reference(args) if args.workload == "mezo" else run_reference_p16(args)
    if args.workload == "p16":
        return run_p16(args)
    if args.workload == "full":
        return run_full(args)

    import torch
    import torch.distributed as dist
    from autoane_b200 import _lib
    from autoane_b200.model import BF16, F16, Config, Model

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    _lib.call("b2p_init", local)
    cfg = Config(dtype=BF16 if args.dtype == "bf16" else F16, max_groups=2 * SEEDS_PER_GPU * SEQS_PER_GPU,
                 lora_ffn=args.lora_ffn,
                 **{k: DIMS[k] for k in ("dim", "hidden", "heads", "kv_heads", "head_dim", "seq", "nlayers", "vocab",
                                         "rank", "rope_theta")})
    model = Model(cfg)
    # the timed CPU reference is the plain (attention-adapter) MeZO step
    keep_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.lora_ffn
    cpu_w = {k: [] for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")} if keep_cpu else None
    for l in range(DIMS["nlayers"]):
        ws = synth_weights(l)
        model.set_layer(l, *ws)
        if keep_cpu:
            for k, w in zip(cpu_w, ws):
                cpu_w[k].append(w)
    embed = synth_embed()
    model.set_embedding(embed, np.arange(N_ACTIVE, dtype=np.int32))
    lay = lora_layout(args.lora_ffn)
    model.set_trainable(synth_theta(lay))
    tokens = token_stream()

    W, K = args.warmup, args.steps
    dev = torch.device("cuda", local)
    stream = torch.cuda.ExternalStream(model.stream)
    # device-resident inputs for every step of the device-timed run
    batches = [step_batch(tokens, s, rank, SEQS_PER_GPU) for s in range(W + K)]
    d_tok = torch.tensor(np.stack([b[0] for b in batches]).astype(np.int32), device=dev)
    d_tgt = torch.tensor(np.stack([b[1] for b in batches]).astype(np.int32), device=dev)
    torch.cuda.synchronize()
    pairs = torch.zeros(2 * SEEDS_PER_GPU, device=dev)
    gathered = torch.zeros(2 * SEEDS_PER_GPU * world, device=dev)

    def dev_step(s):
        seeds = step_seeds(s, world)
        local_seeds = seeds[SEEDS_PER_GPU * rank:SEEDS_PER_GPU * (rank + 1)]
        model.mezo_eval_device(d_tok[s].data_ptr(), d_tgt[s].data_ptr(), SEQS_PER_GPU, local_seeds, float(EPS),
                               pairs.data_ptr())
        if world > 1:
            dist.all_gather_into_tensor(gathered, pairs)
            model.mezo_update(seeds, gathered.data_ptr(), float(EPS), float(LR))
        else:
            model.mezo_update(seeds, pairs.data_ptr(), float(EPS), float(LR))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        for s in range(W):
            dev_step(s)
        model.sync()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        try:
            phys = int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
        except (KeyError, ValueError, IndexError):
            phys = local
        clocks = ClockSampler(phys)
        clocks.start()
        n_launch0 = int(_lib.load().b2p_launch_count())
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for s in range(W, W + K):
            dev_step(s)
        ev1.record(stream)
        model.sync()
        torch.cuda.synchronize()
        n_launch = int(_lib.load().b2p_launch_count()) - n_launch0
        dev_ms = ev0.elapsed_time(ev1)
        barrier()
        clk = clocks.stop()
        # per-GEMM CUDA events of one more step, outside the timed region (their records cost time)
        gemm_ms, gemm_flops, gemm_n = 0.0, 0.0, 0
        if not args.no_profile:
            model.profile(True)
            dev_step(W + K - 1)
            model.sync()
            torch.cuda.synchronize()
            gemm_ms, gemm_flops, gemm_n = model.profile_read()
            model.profile(False)
        barrier()

        # e2e: host buffers through the C ABI, every step copies its inputs in and its losses out
        e_batches = [step_batch(tokens, 10_000 + s, rank, SEQS_PER_GPU) for s in range(K)]
        host_pairs = np.zeros(2 * SEEDS_PER_GPU, np.float32)
        model.sync()
        torch.cuda.synchronize()
        barrier()
        clocks_e2e = ClockSampler(phys)
        clocks_e2e.start()
        t0 = time.perf_counter()
        for s in range(K):
            seeds = step_seeds(10_000 + s, world)
            inp, tgt = e_batches[s]
            model.mezo_eval(inp, tgt, seeds[SEEDS_PER_GPU * rank:SEEDS_PER_GPU * (rank + 1)],
                            float(EPS), out=host_pairs)
            if world > 1:
                pairs.copy_(torch.from_numpy(host_pairs))
                dist.all_gather_into_tensor(gathered, pairs)
                model.mezo_update(seeds, gathered.data_ptr(), float(EPS), float(LR))
            else:
                model.mezo_update(seeds, host_pairs, float(EPS), float(LR))
        model.sync()
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - t0
        clk_e2e = clocks_e2e.stop()
        barrier()
        ranks = rank_checks(model, dev_ms, K, world, dev)

    # max over ranks
    t = torch.tensor([dev_ms, e2e_s, gemm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s, gemm_ms_max = t.tolist()
    units = SEQS_PER_GPU * SEEDS_PER_GPU * world * K
    value = units / (dev_ms / 1000.0)
    e2e_value = units / e2e_s

    roofline = None
    if gemm_n:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        peak = peaks.get("bf16_tflops_sustained")
        peak_src = "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)"
        if peak is None:
            peak, peak_src = 1400.0, "fallback sustained 1.4 PFLOP/s"
        achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "traffic": gemm_traffic_per_launch(),
                    "kernel": "gemm_pair_kernel (projection + lm-head launches of one step after the timed region)",
                    "launches": gemm_n,
                    "avg_launch_us": round(1000.0 * gemm_ms / gemm_n, 2), "peak_source": peak_src,
                    "flops_per_launch_avg": gemm_flops / gemm_n}
    h2d = 2 * SEQS_PER_GPU * DIMS["seq"] * 4 + 2 * cfg.max_groups * 4 + 2 * SEEDS_PER_GPU * 16 + \
        SEEDS_PER_GPU * 8 + SEEDS_PER_GPU * world * 8 + (0 if world > 1 else 2 * SEEDS_PER_GPU * 4)
    d2h = 2 * SEEDS_PER_GPU * 4
    if rank == 0:
        cpu = None
        if keep_cpu:
            cpu = cpu_reference_rate(weights=cpu_w, embed=embed)
            one = cpu_reference_rate(max_seconds=25.0, max_steps=3, min_steps=1, weights=cpu_w, embed=embed, threads=1)
            logical, physical = host_cores()
            cpu |= {"cores_logical": logical, "cores_physical": physical,
                    "one_core": {"value": one["value"], "unit": one["unit"], "cores": 1, "sample": one["sample"]}}
        line = {"metric": "MeZO-LoRA steps/s SmolLM2-360M @1/2/4/8 B200; proj-GEMM % of TC peak",
                "value": round(value, 3), "unit": "seq-steps/s", "n_gpus": world, "steps": K, "warmup": W,
                "ms_per_step": round(dev_ms / K, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": round(value / REF_STEPS_PER_S, 2), "dtype": args.dtype, "data": "synthetic",
                "config": workload_config(world, args.lora_ffn) | {
                    "optimizer_steps_per_s": round(K / (dev_ms / 1000.0), 3),
                    "tflops_per_gpu": round(2 * SEQS_PER_GPU * SEEDS_PER_GPU * fwd_flops_per_seq(args.lora_ffn) * K /
                                            (dev_ms / 1000.0) / 1e12, 2)},
                "e2e": {"value": round(e2e_value, 3), "unit": "seq-steps/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h,
                        "sm_mhz": clk_e2e["sm_mhz"] if clk_e2e else None},
                "gpu_launches": n_launch, "roofline": roofline, "clocks": clk, "cpu_baseline": cpu}
        if ranks:
            line["ranks"] = ranks
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()
    if ranks and not ranks["theta_identical_across_ranks"]:
        print("ERROR: the trainable parameters differ between ranks", file=sys.stderr)
        return 1
    return 0


# --------------------------------------------------------------------------- backprop-LoRA (P16) workload
P16_SEQS_PER_GPU = 8
P16_LR = 3e-4
REF_P16_MS = 612.0  # reference P16 CPU step (fwd 234 + bwd 360 + opt 18 ms, results/p16_backprop_lora_cpu_200steps.txt)


def p16_flops_per_seq() -> float:
    """Algorithmic FLOPs of one P16 sequence step: forward + dX of the 7 projections + classifier backward
    (logit recompute + dy) + attention backward (4 dense T^2 matmuls + score recompute) + factored dA/dB."""
    d = DIMS
    s, D, H, r, L = d["seq"], d["dim"], d["hidden"], d["rank"], d["nlayers"]
    qd, kvd = d["heads"] * d["head_dim"], d["kv_heads"] * d["head_dim"]
    proj = 2 * s * (D * (qd + 2 * kvd) + qd * D + 3 * D * H)
    attn_mm = 2 * d["heads"] * s * s * d["head_dim"]
    head = 2 * s * N_ACTIVE * D
    lora_grad = 2 * s * r * 2 * ((qd + 2 * kvd) + D + 3 * D + qd)
    bwd = L * (proj + 5 * attn_mm + lora_grad) + 2 * head
    return fwd_flops_per_seq() + float(bwd)


def p16_config(world: int, nseq: int = P16_SEQS_PER_GPU):
    return {"workload": f"DP backprop-LoRA (P16) r8, SmolLM2-360M shapes, SEQ 256; per GPU {nseq} sequences, "
                        "forward + full backward + NCCL all-reduce of the LoRA/RMS gradient + Adam",
            "model": "SmolLM2-360M-shaped (random init)", "global_batch": nseq * world,
            "seq_len": DIMS["seq"], "parallelism": f"dp{world}", "lora_rank": DIMS["rank"], "lr": P16_LR,
            "adam": "b1 0.9, b2 0.95, eps 1e-8, wd 0", "l2": "inputs larger than L2 (1.3 GB of weights per step)",
            "gflop_per_seq_step": round(p16_flops_per_seq() / 1e9, 2)}


def run_p16(args):
    import torch
    import torch.distributed as dist
    from autoane_b200 import _lib
    from autoane_b200.model import BF16, F16, Config, Model

    rank, world, local = env_rank()
    NSEQ = args.p16_seqs
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    _lib.call("b2p_init", local)
    cfg = Config(dtype=BF16 if args.dtype == "bf16" else F16, max_groups=NSEQ,
                 **{k: DIMS[k] for k in ("dim", "hidden", "heads", "kv_heads", "head_dim", "seq", "nlayers", "vocab",
                                         "rank", "rope_theta")})
    model = Model(cfg)
    for l in range(DIMS["nlayers"]):
        model.set_layer(l, *synth_weights(l))
    embed = synth_embed()
    model.set_embedding(embed, np.arange(N_ACTIVE, dtype=np.int32))
    model.set_trainable(synth_theta(lora_layout()))
    tokens = token_stream()
    W, K = args.warmup, args.steps
    dev = torch.device("cuda", local)
    stream = torch.cuda.ExternalStream(model.stream)
    batches = [step_batch(tokens, s, rank, NSEQ) for s in range(W + K)]
    d_tok = torch.tensor(np.stack([b[0] for b in batches]).astype(np.int32), device=dev)
    d_tgt = torch.tensor(np.stack([b[1] for b in batches]).astype(np.int32), device=dev)
    d_loss = torch.zeros(1, device=dev)
    torch.cuda.synchronize()

    def grad_tensor():
        class _G:  # the model's device gradient buffer as a torch tensor (no copy)
            __cuda_array_interface__ = {"shape": (model.P,), "typestr": "<f4", "data": (model.grad_ptr(), False),
                                        "version": 3, "stream": None}
        return torch.as_tensor(_G(), device=dev)

    grad = None

    def allreduce():
        if world > 1:
            dist.all_reduce(grad)
            grad.mul_(1.0 / world)

    def dev_step(s):
        nonlocal grad
        model.p16_grad_device(d_tok[s].data_ptr(), d_tgt[s].data_ptr(), NSEQ, d_loss.data_ptr())
        if grad is None:
            grad = grad_tensor()
        allreduce()
        model.adam_step(P16_LR)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        for s in range(W):
            dev_step(s)
        model.sync()
        torch.cuda.synchronize()
        barrier()
        try:
            phys = int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
        except (KeyError, ValueError, IndexError):
            phys = local
        clocks = ClockSampler(phys)
        clocks.start()
        n_launch0 = int(_lib.load().b2p_launch_count())
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for s in range(W, W + K):
            dev_step(s)
        ev1.record(stream)
        model.sync()
        torch.cuda.synchronize()
        n_launch = int(_lib.load().b2p_launch_count()) - n_launch0
        dev_ms = ev0.elapsed_time(ev1)
        barrier()
        clk = clocks.stop()
        # per-GEMM CUDA events of one more step (its graph holds the event records; not in the timed region)
        gemm_ms, gemm_flops, gemm_n = 0.0, 0.0, 0
        if not args.no_profile:
            model.profile(True)
            dev_step(W + K - 1)
            dev_step(W + K - 1)
            model.sync()
            gemm_ms, gemm_flops, gemm_n = model.profile_read()
            model.profile(False)
            barrier()
        # e2e through the host-buffer C ABI: tokens in, loss out, every step
        e_batches = [step_batch(tokens, 20_000 + s, rank, NSEQ) for s in range(K)]
        model.sync()
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        last = 0.0
        for s in range(K):
            inp, tgt = e_batches[s]
            if world > 1:
                last, _ = model.p16_grad(inp, tgt)
                allreduce()
                model.adam_step(P16_LR)
            else:
                last = model.p16_step(inp, tgt, P16_LR)
        model.sync()
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - t0
        barrier()
        ranks = rank_checks(model, dev_ms, K, world, dev)
    t = torch.tensor([dev_ms, e2e_s, gemm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s, gemm_ms = t.tolist()
    units = NSEQ * world * K
    value = units / (dev_ms / 1000.0)
    roofline = None
    if gemm_n:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        peak = peaks.get("bf16_tflops_sustained", 1400.0)
        achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "traffic": None,
                    "kernel": "tcgen05 GEMMs (forward + data-gradient launches) of the last step (CUDA graph)",
                    "launches": gemm_n,
                    "avg_launch_us": round(1000.0 * gemm_ms / gemm_n, 2),
                    "peak_source": "measured sustained cuBLAS bf16 (MEASURED_PEAKS.json)"}
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_reference_p16_rate()
        line = {"metric": "backprop-LoRA (P16) seq-steps/s SmolLM2-360M", "value": round(value, 3),
                "unit": "seq-steps/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(dev_ms / K, 4),
                "higher_is_better": True, "scaling": "weak",
                "vs_baseline": round(value / (1000.0 / REF_P16_MS), 2), "dtype": args.dtype, "data": "synthetic",
                "config": p16_config(world, NSEQ) | {
                    "tflops_per_gpu": round(NSEQ * p16_flops_per_seq() * K / (dev_ms / 1000.0) / 1e12, 2),
                    "last_e2e_loss": round(float(last), 5)},
                "e2e": {"value": round(units / e2e_s, 3), "unit": "seq-steps/s",
                        "h2d_bytes_per_step": 2 * NSEQ * DIMS["seq"] * 4 + 2 * cfg.max_groups * 4 + 16,
                        "d2h_bytes_per_step": 4},
                "gpu_launches": n_launch, "roofline": roofline, "clocks": clk, "cpu_baseline": cpu}
        if ranks:
            line["ranks"] = ranks
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()
    if ranks and not ranks["theta_identical_across_ranks"]:
        print("ERROR: the trainable parameters differ between ranks", file=sys.stderr)
        return 1
    return 0


def _ref_p16_fn():
    """(callable running one reference P16 gradient step on SmolLM2 shapes, threads) or None."""
    from oracle import oracle as O
    import ctypes as C
    ref = O.ref_lib("smollm2_360m")
    if ref is None:
        return None
    rng = np.random.default_rng(0)
    L, D, H = DIMS["nlayers"], DIMS["dim"], DIMS["hidden"]
    qd, kvd, r = DIMS["heads"] * 64, DIMS["kv_heads"] * 64, DIMS["rank"]
    F = C.POINTER(C.c_float)
    keep = []

    def f(a):
        return a.ctypes.data_as(F)

    def plist(arrs):
        p = (F * len(arrs))(*[f(a) for a in arrs])
        keep.append((arrs, p))
        return p
    ws = [synth_weights(l) for l in range(L)]
    Wl = [plist([w[i] for w in ws]) for i in range(7)]
    sizes = [r * D, qd * r, r * D, kvd * r, r * D, kvd * r, r * qd, D * r]
    lora = [(0.1 * rng.standard_normal(sizes[k % 8])).astype(np.float32) for k in range(8 * L)]
    rms = [np.ones(D, np.float32) for _ in range(2 * L)]
    rf = np.ones(D, np.float32)
    embed = synth_embed()
    cembed = np.ascontiguousarray(embed[:N_ACTIVE])
    glora = [np.zeros(sizes[k % 8], np.float32) for k in range(8 * L)]
    grms = [np.zeros(D, np.float32) for _ in range(2 * L)]
    grf = np.zeros(D, np.float32)
    tokens = token_stream()
    inp, tgt = step_batch(tokens, 0, 0, 1)
    inp, tgt = np.ascontiguousarray(inp[0], np.uint16), np.ascontiguousarray(tgt[0], np.uint16)
    ref.ref_p16_grad.argtypes = [C.POINTER(F)] * 9 + [F, F, F, C.c_int, C.c_int, C.c_float,
                                                      C.POINTER(C.c_uint16), C.POINTER(C.c_uint16),
                                                      C.POINTER(F), C.POINTER(F), F]
    args = (*Wl, plist(lora), plist(rms), f(rf), f(embed), f(cembed), N_ACTIVE, r, C.c_float(1.0),
            inp.ctypes.data_as(C.POINTER(C.c_uint16)), tgt.ctypes.data_as(C.POINTER(C.c_uint16)), plist(glora),
            plist(grms), f(grf))
    mom = [np.zeros(a.size, np.float32) for a in lora]
    vel = [np.zeros(a.size, np.float32) for a in lora]

    def step():
        _ = keep  # the arrays behind the pointer lists must outlive the calls
        ref.ref_p16_grad(*args)
        for k in range(8 * L):  # the reference's Adam on every LoRA buffer (train_mezo.m:2099-2106)
            ref.ref_adam(f(lora[k]), f(glora[k]), f(mom[k]), f(vel[k]), C.c_size_t(lora[k].size), 1,
                         C.c_float(P16_LR), C.c_float(0.9), C.c_float(0.95), C.c_float(1e-8), C.c_float(0.0))
    return step, O.set_threads(os.cpu_count() or 1)


def cpu_reference_p16_rate(max_seconds: float = 30.0):
    got = _ref_p16_fn()
    if got is None:
        return None
    step, threads = got
    t0 = time.perf_counter()
    n = 0
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 > max_seconds / 2 or n >= 3:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": "seq-steps/s", "cores": threads, "kind": "reference",
            "sample": f"{n} P16 steps (batch 1, SEQ 256) of the reference's forward transcription + compiled "
                      "bp_lora_backward + adam_update, OpenBLAS"}


def run_reference_p16(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    r = cpu_reference_p16_rate(max_seconds=max(30.0, 10.0 * args.steps))
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref_smollm2_360m.so was not built"}))
        return 0
    print(json.dumps({"impl": "reference", "metric": "backprop-LoRA (P16) seq-steps/s SmolLM2-360M",
                      "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
                      "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "dtype": "f32",
                      "data": "synthetic", "config": p16_config(world), "cpu_baseline": r,
                      "e2e": {"value": r["value"], "unit": r["unit"], "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)
    return 0


# --------------------------------------------------------------------------- full backprop (config 0)
AR_DIMS = dict(dim=512, hidden=1408, heads=8, kv_heads=2, head_dim=64, seq=128, nlayers=4, vocab=49152, rank=8,
               rope_theta=10000.0)  # training/models/autoresearch.h
REF_FULL_MS = 24.0  # reference train.m CPU step on the autoresearch model (FINDINGS.md:94)


def full_flops_per_seq() -> float:
    """Projection FLOPs of one train.m step per sequence: forward + dX + dW of the 7 projections and the
    compact classifier (3 x forward)."""
    d = AR_DIMS
    s, D, H = d["seq"], d["dim"], d["hidden"]
    qd, kvd = d["heads"] * d["head_dim"], d["kv_heads"] * d["head_dim"]
    per_layer = D * (qd + 2 * kvd) + qd * D + 3 * D * H
    return 3.0 * (d["nlayers"] * 2 * s * per_layer + 2 * s * N_ACTIVE * D)


def ar_synth(layer: int):
    rng = np.random.default_rng([4242, layer])
    D, H = AR_DIMS["dim"], AR_DIMS["hidden"]
    qd, kvd = AR_DIMS["heads"] * AR_DIMS["head_dim"], AR_DIMS["kv_heads"] * AR_DIMS["head_dim"]
    shapes = [(qd, D), (kvd, D), (kvd, D), (D, qd), (H, D), (D, H), (H, D)]
    return [rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02) for sh in shapes]


def run_full(args):
    import torch
    from autoane_b200 import _lib
    from autoane_b200.model import BF16, F16, Config, Model
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    _lib.call("b2p_init", local)
    NSEQ = args.full_seqs
    cfg = Config(dtype=BF16 if args.dtype == "bf16" else F16, max_groups=NSEQ, **AR_DIMS)
    model = Model(cfg)
    ws = [ar_synth(l) for l in range(AR_DIMS["nlayers"])]
    for l in range(AR_DIMS["nlayers"]):
        model.set_layer(l, *ws[l])
    rng = np.random.default_rng([4242, 99])
    embed = (rng.standard_normal((AR_DIMS["vocab"], AR_DIMS["dim"]), dtype=np.float32) * 0.02).astype(np.float32)
    model.set_embedding(embed, np.arange(N_ACTIVE, dtype=np.int32))
    D, r, L = AR_DIMS["dim"], AR_DIMS["rank"], AR_DIMS["nlayers"]
    qd, kvd = AR_DIMS["heads"] * 64, AR_DIMS["kv_heads"] * 64
    theta = np.zeros(model.P, np.float32)
    per = [r * D, qd * r, r * D, kvd * r, r * D, kvd * r, r * qd, D * r, D, D]
    o = 0
    for l in range(L):
        for k, n in enumerate(per):
            if k >= 8:
                theta[o:o + n] = 1.0  # RMS weights; LoRA B = 0 so the adapters do not act
            elif k % 2 == 0:
                theta[o:o + n] = rng.standard_normal(n).astype(np.float32) / np.sqrt(r)
            o += n
    theta[o:o + D] = 1.0
    model.set_trainable(theta)
    tokens = token_stream()
    W, K = args.warmup, args.steps
    seq = AR_DIMS["seq"]

    def batch(step):
        g = np.random.default_rng([7919, step, rank])
        pos = g.integers(0, int(len(tokens) * 0.9) - seq - 1, NSEQ)
        return (np.stack([tokens[p:p + seq] for p in pos]), np.stack([tokens[p + 1:p + 1 + seq] for p in pos]))
    batches = [batch(s) for s in range(W + K)]
    stream = torch.cuda.ExternalStream(model.stream)
    for s in range(W):
        model.full_step(*batches[s], 3e-4, 0.1, 1.0)
    torch.cuda.synchronize()
    try:
        phys = int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    except (KeyError, ValueError, IndexError):
        phys = local
    clocks = ClockSampler(phys)
    clocks.start()
    n0 = int(_lib.load().b2p_launch_count())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    t0 = time.perf_counter()
    last = (0.0, 0.0)
    for s in range(W, W + K):
        last = model.full_step(*batches[s], 3e-4, 0.1, 1.0)
    ev1.record(stream)
    torch.cuda.synchronize()
    host_s = time.perf_counter() - t0
    dev_ms = ev0.elapsed_time(ev1)
    n_launch = int(_lib.load().b2p_launch_count()) - n0
    clk = clocks.stop()
    units = NSEQ * K
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_full_rate(ws, embed, theta, tokens)
        line = {"metric": "full-backprop (train.m) seq-steps/s, autoresearch 36.4M (4L d512 8/2 heads FFN 1408) T128",
                "value": round(units / (dev_ms / 1000.0), 3), "unit": "seq-steps/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": round(dev_ms / K, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": round(units / (dev_ms / 1000.0) / (1000.0 / REF_FULL_MS), 2), "dtype": args.dtype,
                "data": "synthetic",
                "config": {"workload": f"full backprop, per GPU {NSEQ} x 128-token sequences per step; forward, dX and "
                                       "dW of every projection, tied-embedding gradient, global-norm clip 1.0, AdamW "
                                       "(lr 3e-4, wd 0.1); replicas on N > 1 GPUs", "model": "autoresearch-4L-512d",
                           "global_batch": NSEQ * world, "seq_len": seq, "parallelism": f"replicas x{world}",
                           "tflops_per_gpu": round(NSEQ * full_flops_per_seq() * K / (dev_ms / 1000.0) / 1e12, 2),
                           "last_loss": round(float(last[0]), 5), "last_grad_norm": round(float(last[1]), 5),
                           "inputs": "host tokens staged every step (16 KB H2D incl. the per-token segment table)"},
                "e2e": {"value": round(units / host_s, 3), "unit": "seq-steps/s",
                        "h2d_bytes_per_step": NSEQ * seq * 2 * 4 + (2 * NSEQ * seq + 2) * 4,
                        "d2h_bytes_per_step": 8},
                "gpu_launches": n_launch, "roofline": None, "clocks": clk, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    model.close()
    return 0


def cpu_full_rate(ws, embed, theta, tokens, max_seconds: float = 20.0):
    """The oracle's train.m step (or_full_grad + adam_update), batch 1, on this host's cores."""
    from oracle import oracle as O
    threads = O.set_threads(os.cpu_count() or 1)
    cfg = O.ModelCfg(dim=AR_DIMS["dim"], hidden=AR_DIMS["hidden"], heads=AR_DIMS["heads"],
                     kv_heads=AR_DIMS["kv_heads"], hd=64, seq=AR_DIMS["seq"], nlayers=AR_DIMS["nlayers"],
                     vocab=AR_DIMS["vocab"], rank=AR_DIMS["rank"], rope_theta=AR_DIMS["rope_theta"])
    weights = {k: [w[i] for w in ws] for i, k in enumerate(("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3"))}
    om = O.OracleModel(cfg, weights, embed, np.ascontiguousarray(embed[:N_ACTIVE]))
    seq = AR_DIMS["seq"]
    n, t0 = 0, time.perf_counter()
    while n < 3 or (time.perf_counter() - t0 < max_seconds and n < 200):
        p = (n * 7919) % (len(tokens) - seq - 2)
        loss, g, dw, ge = om.full_grad(theta, tokens[p:p + seq], tokens[p + 1:p + 1 + seq])
        flat = np.concatenate([a.ravel() for k in dw for a in dw[k]])
        zeros = np.zeros_like(flat)
        O.adam(flat, flat.copy(), zeros, zeros.copy(), 1, 3e-4, wd=0.1)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "seq-steps/s", "cores": threads, "kind": "port",
            "sample": f"{n} train.m steps (batch 1, T 128) of the oracle restatement (or_full_grad + adam_update over "
                      "the projection weights), OpenBLAS; the reference's train.m is Objective-C and does not build here"}


# --------------------------------------------------------------------------- projection-GEMM sweep
GEMM_SHAPES = {"Wq": (960, 960), "Wk/Wv": (320, 960), "Wo": (960, 960), "W1/W3": (2560, 960), "W2": (960, 2560),
               "lm_head": (49152, 960), "lm_head_compact": (16893, 960)}


def run_gemm_sweep(args):
    """Y[T, M] = X[T, K] · W[M, K]^T on the tcgen05 engine for every (shape, T) of the projection sweep;
    one JSON line per case with TFLOP/s and the HBM/tensor roofline of that shape."""
    import torch
    from autoane_b200 import _lib
    _, _, local = env_rank()
    torch.cuda.set_device(local)
    _lib.call("b2p_init", local)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tc = peaks.get("bf16_tflops", 1590.0)
    bw = peaks.get("hbm_gbs", 6650.0)
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    code = 1 if args.dtype == "bf16" else 0
    dev = torch.device("cuda", local)
    flush = None
    del flush
    for name, (M, K) in GEMM_SHAPES.items():
        for T in (128, 256, 1024, 8192):
            # enough operand copies that one pass over them exceeds L2 (126 MB): every launch reads from HBM
            per = 2 * (T * K + M * K) + 4 * T * ((M + 3) // 4 * 4) + 4 * T * ((M + 7) // 8 * 8)
            ncopy = max(2, min(64, -(-(256 << 20) // per)))
            xs = [torch.randn(T, K, device=dev).to(dt) for _ in range(ncopy)]
            ws = [(0.02 * torch.randn(M, K, device=dev)).to(dt) for _ in range(ncopy)]
            ys = [torch.empty(T, (M + 3) // 4 * 4, device=dev, dtype=torch.float32) for _ in range(ncopy)]
            hs = [torch.empty(T, (M + 7) // 8 * 8, device=dev, dtype=dt) for _ in range(ncopy)]
            # cuBLAS gets the same 8-element-aligned output rows as the engine (W zero-padded to M8 rows):
            # an odd leading dimension would put it on a slow unaligned path
            M8 = (M + 7) // 8 * 8
            wc = [torch.cat([w, torch.zeros(M8 - M, K, device=dev, dtype=dt)]) if M8 > M else w for w in ws]
            cs = [torch.empty(T, M8, device=dev, dtype=dt) for _ in range(ncopy)]
            # up to 1024 rows b2p_gemm splits each tile's K loop over a cluster; above, the CTA-pair engine
            fn = "b2p_gemm" if T <= 1024 else "b2p_gemm_pair"

            def ours(i, f32=True):
                st = torch.cuda.current_stream().cuda_stream
                y = ys[i] if f32 else hs[i]
                _lib.call(fn, xs[i].data_ptr(), ws[i].data_ptr(), y.data_ptr(), T, M, K, y.shape[1], code,
                          1 if f32 else 0, st)

            def cublas(i):  # the library baseline: cuBLAS through torch, 16-bit output
                torch.mm(xs[i], wc[i].t(), out=cs[i])

            def graph_ms(run):
                for i in range(ncopy):
                    run(i)
                torch.cuda.synchronize()
                # back-to-back launches over the rotating copies, recorded once into a CUDA graph so
                # the host's per-call cost stays out of the timed region
                reps = max(ncopy, 8 * max(5, args.steps))
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for i in range(reps):
                        run(i % ncopy)
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                del graph
                return e0.elapsed_time(e1) / reps, reps

            ms, reps = graph_ms(ours)
            ms16, _ = graph_ms(lambda i: ours(i, False))
            msc, _ = graph_ms(cublas)
            flops = 2.0 * M * K * T
            byts = 2.0 * M * K + 2.0 * K * T + 4.0 * M * T
            roof = min(tc, bw * 1e9 * flops / byts / 1e12)
            ach = flops / (ms / 1000.0) / 1e12
            print(json.dumps({"metric": "projection GEMM TFLOP/s", "shape": name, "M": M, "K": K, "T": T,
                              "dtype": args.dtype, "value": round(ach, 2), "unit": "TFLOP/s", "us": round(ms * 1e3, 2),
                              "roofline_tflops": round(roof, 1), "frac_of_roofline": round(ach / roof, 3),
                              "bound": "tensor" if roof >= tc else "hbm", "engine": fn,
                              "us_16bit_out": round(ms16 * 1e3, 2), "cublas_us_16bit_out": round(msc * 1e3, 2),
                              "l2": f"operands rotate over {ncopy} copies (> 256 MB) so every launch reads HBM",
                              "timing": f"{reps} back-to-back launches in one CUDA graph, CUDA events"}),
                  flush=True)
            del xs, ws, ys, hs, cs, wc
    return 0


def gemm_traffic_per_launch():
    """DRAM bytes per projection-GEMM launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "gemm_pair_kernel_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


if __name__ == "__main__":
    sys.exit(main())
