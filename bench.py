#!/usr/bin/env python
"""Benchmark of the DWA hot path on B200: retrieve + gather + assemble, the
pool and its IVF lists row-sharded over the GPUs of one node.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
                    [--workload medium|small|large|decode]

Default workload ``medium``: bf16, global batch 16, seq 1024, d 2048, pool
1M x 34816 rows (73 GB), 1024 lists, nprobe 16, top-k 64, gate selection with
soft_full, forward.  Rank p of N holds the rows of a contiguous run of whole
lists and their keys; one step is the sequence means of its sequences, an
all-gather of z, ``dwa_retrieve_local`` over its rows, an all-gather of the
[B, 2k+3] summaries, ``dwa_retrieve_merge``, the winning rows of its
sequences read from their owners by peer loads (``dwa_gather_rows``) and
``dwa_assemble_fwd`` of its B/N sequences.  Strong scaling: the job is the
same at every N.  ``value`` is the job's assembled tokens/s: B*T over the step
time, timed on the device with CUDA events around each step (a barrier before
every step, L2 flushed between steps, the per-step maximum over ranks).

At N=1 the line also carries ``small_fwd_bwd`` (the single-GPU small workload,
forward + custom-VJP backward), the key-cache GEMM, the retrieval VJP, the aux
losses and ``cpu_baseline``.  ``parity`` compares the sharded result with the
single-device call over the all-gathered key cache and the peer-read rows with
the masked-psum gather of the reference's model-sharded path.

``--impl reference`` times the reference's algorithm on the host CPU: the
NumPy restatement of the reference (JAX is not installable here), batched as
the reference calls it, on all host cores, no GPU and nothing of this
package.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "assembled tokens/sec/GPU (retrieve+assemble+apply) at 1/2/4/8 B200; % HBM/tensor roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_NOTE = "flushed between steps (512 MB write, then 256 MB read)"
ROWS_WORKLOADS = ("medium", "large")

# The workloads' sizes, restated for the host-only reference arm (which
# imports nothing of the package); tests/test_bench_cpu.py checks them against
# matrix_b200.config.WORKLOADS.  sample_B: sequences per reference step.
HOST_WORKLOADS = {
    "small": dict(B=8, T=512, d=1024, N=262144, C=512, m=8, k=32, r=8, S=4, dk=64, zipf=None,
                  backward=True, soft_full=True, lam=5.0, warmup=False, sample_B=4),
    "medium": dict(B=16, T=1024, d=2048, N=1 << 20, C=1024, m=16, k=64, r=8, S=4, dk=64, zipf=None,
                   backward=False, soft_full=True, lam=5.0, warmup=False, sample_B=2),
    "large": dict(B=32, T=2048, d=2048, N=1 << 22, C=4096, m=32, k=64, r=8, S=4, dk=64, zipf=1.1,
                  backward=True, soft_full=True, lam=5.0, warmup=False, sample_B=1),
}
NOTES = {
    "small": "bf16, batch 8, seq 512, d 1024, pool 262144, 512 lists, nprobe 8, top-k 32, fwd+bwd",
    "medium": "bf16, batch 16, seq 1024, d 2048, pool 1M, 1024 lists, nprobe 16, top-k 64, fwd",
    "large": "bf16, batch 32, seq 2048, d 2048, pool 4M, 4096 Zipf(1.1) lists, nprobe 32, top-k 64",
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="medium")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget-s", type=float, default=20.0,
                    help="CPU seconds for the cpu_baseline sample (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sharded", action="store_true",
                    help="row-shard the pool of the small workload too (medium and large always are)")
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="row-sharded, one GPU: run the rank of this many that holds the most rows (its row "
                         "share, retrieval of the whole batch over it, assembly of its sequences), no collectives")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-small", action="store_true", help="skip the small fwd+bwd extra at N=1")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip timing the retrieval VJP and the auxiliary losses")
    ap.add_argument("--no-key-cache", action="store_true",
                    help="skip timing compute_key_cache (once per window, not part of the step)")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="for an ncu launch list: after one warm-up step, run this many eager steps, each "
                         "inside an NVTX range 'dwa_step' (an L2 flush before each, outside it), then exit")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return FALLBACK_PEAKS, "fallback"


def step_description(name, rows_mode, world, backward, emulate=0):
    if rows_mode:
        gather = ("dwa_gather_rows (peer loads of the winning rows)" if world > 1 or emulate else
                  "winning rows read from the pool by index inside the assembly")
        retr = ("all-gather of z + dwa_retrieve_local + all-gather of summaries + dwa_retrieve_merge"
                if world > 1 else "dwa_retrieve_local + dwa_retrieve_merge" if emulate else "dwa_retrieve")
        s = "CUDA graph: seq_mean + " + retr + " + " + gather + (
            " + dwa_assemble_apply (h_mid only)" if name == "decode" else " + dwa_assemble_fwd")
        if backward:
            s += (" + dwa_assemble_bwd + pool-row gradients to their owners (peer stores of bf16 rows) and "
                  "scatter" +
                  (" + NCCL all_reduce of parameter grads" if world > 1 else ""))
        return s
    return ("CUDA graph: seq_mean + dwa_retrieve + dwa_assemble_fwd" + (" + dwa_assemble_bwd" if backward else "")
            + (" + NCCL all_reduce of parameter grads" if world > 1 and backward else ""))


def run_config(name, world, rows_mode, emulate=0, w=None):
    """The ``config`` object of the JSON line; identical for both arms.  A
    workload without a host restatement (the ncu cases) takes its sizes from
    ``w``."""
    if name in HOST_WORKLOADS:
        h, note = HOST_WORKLOADS[name], NOTES[name]
    else:
        h = dict(B=w.batch, T=w.seq, warmup=w.is_warmup, lam=w.lambda_val, soft_full=w.soft_full,
                 backward=w.backward)
        note = w.note
    cfg = {"workload": name, "note": note,
           "global_batch": h["B"] if rows_mode else h["B"] * world, "seq_len": h["T"],
           "parallelism": (f"rows{emulate}, one rank emulated on one GPU" if emulate
                           else f"rows{world}" if rows_mode else f"dp{world}"),
           "mode": "warmup" if h["warmup"] else f"gate lambda={h['lam']}",
           "soft_full": h["soft_full"], "backward": h["backward"], "l2": L2_NOTE,
           "step": step_description(name, rows_mode, world, h["backward"], emulate)}
    return cfg


# ======================================================================
# Host reference arm: the reference's algorithm on the CPU (NumPy port)
# ======================================================================
def _zipf_offsets(N, C, s, rng):
    w = 1.0 / np.arange(1, C + 1, dtype=np.float64) ** s
    sizes = np.floor(w / w.sum() * (N - C)).astype(np.int64) + 1
    sizes[0] += N - sizes.sum()
    rng.shuffle(sizes)
    off = np.zeros(C + 1, dtype=np.int64)
    np.cumsum(sizes, out=off[1:])
    return off


def host_inputs(name, seed, n_pool_rows=4096):
    """Seeded host inputs of workload ``name`` for the reference's CPU path:
    the key cache [S, N, d_k] f32 drawn from N(0, 1/d) (the distribution
    compute_key_cache gives for pool rows ~ N(0, 1/sqrt d) and key projections
    ~ N(0, 1/sqrt D); the 73 GB pool itself is not formed on the host),
    centroids = keys of a random row per list, the retrieval and assembly
    parameters at their initialisation scales, ``sample_B`` sequences of h_A,
    and ``n_pool_rows`` pool rows that the gather reads (row i mod n)."""
    h = HOST_WORKLOADS[name]
    rng = np.random.default_rng(seed)
    d, N, S, dk, C, r, Bs, T = h["d"], h["N"], h["S"], h["dk"], h["C"], h["r"], h["sample_B"], h["T"]
    D = d * (2 * r + 1)
    f32 = np.float32
    keys = rng.standard_normal((S, N, dk), dtype=f32)
    keys *= f32(d ** -0.5)
    off = (_zipf_offsets(N, C, h["zipf"], rng) if h["zipf"] else np.arange(C + 1, dtype=np.int64) * (N // C))
    rows_c = off[:-1] + (rng.random(C) * np.diff(off)).astype(np.int64)
    x = dict(keys=keys, list_offsets=off, centroids=np.ascontiguousarray(keys[:, rows_c, :]),
             W_Q=rng.standard_normal((S, dk, d), dtype=f32) * f32(d ** -0.5),
             aspect_weights=np.zeros(S, f32), tau=f32(0.0),
             W_base=rng.standard_normal((d, d), dtype=f32) * f32(0.01), b_base=np.zeros(d, f32),
             gamma=f32(0.1), h_A=rng.standard_normal((Bs, T, d), dtype=f32),
             pool_rows=rng.standard_normal((n_pool_rows, D), dtype=f32) * f32(d ** -0.5))
    if h["backward"]:
        x["g_hmid"] = rng.standard_normal((Bs, T, d), dtype=f32) * f32(0.1)
        x["g_W"] = rng.standard_normal((Bs, d, d), dtype=f32) * f32(1e-3)
    return x


def host_step(name, x):
    """One batched call of the reference's forward (retrieve + gather + float32
    cast + assemble_jax) and, when the workload has one, its VJP, over the
    ``sample_B`` sequences of ``x``, through the NumPy restatement."""
    from oracle import dwa_oracle as O
    h = HOST_WORKLOADS[name]
    z = x["h_A"].mean(axis=1, dtype=np.float32)
    alphas, idx, _ = O.retrieve(z, x["W_Q"], x["aspect_weights"], x["tau"], x["centroids"], x["keys"],
                                k=h["k"], m=h["m"], T=1.0, lambda_val=h["lam"], is_warmup=h["warmup"],
                                list_offsets=x["list_offsets"], want_soft_full=h["soft_full"])
    gathered = O.gather(x["pool_rows"], idx % x["pool_rows"].shape[0])
    h_mid, W = O.assemble(gathered, alphas, x["h_A"], x["W_base"], x["b_base"], x["gamma"], h["d"], h["r"], h["d"])
    if h["backward"]:
        O.assemble_bwd(gathered, alphas, x["h_A"], W, x["gamma"], x["g_hmid"], x["g_W"], h["d"], h["r"], h["d"])
    return h_mid


def host_threads():
    """Let every BLAS / OpenMP pool use all host cores (torchrun sets
    OMP_NUM_THREADS=1 on every rank); returns (os.cpu_count(), threads in use)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n)
        used = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        used = 1
    return n, used


def host_sample_desc(name):
    h = HOST_WORKLOADS[name]
    return (f"batched call over {h['sample_B']} of the {h['B']} sequences per step ({h['T']} tokens each): "
            f"retrieve over all {h['N']} key rows (IVF {h['C']} lists, nprobe {h['m']}, top-k {h['k']}, "
            f"{'soft_full, ' if h['soft_full'] else ''}gate lambda {h['lam']}), gather + float32 cast, "
            f"assemble_jax{' + its VJP' if h['backward'] else ''}; NumPy float32 restatement of "
            f"retrieval.py:48-159, model.py:193-195, assembly_pallas.py:42-75"
            f"{', 246-329' if h['backward'] else ''}; keys drawn from the compute_key_cache distribution, "
            f"gathered rows from a 4096-row host pool")


def reference_arm(args, rank, world):
    """--impl reference: rank 0 times the host path; other ranks exit at once."""
    if rank != 0:
        return
    name = args.workload
    if name not in HOST_WORKLOADS:
        print(json.dumps({"impl": "reference", "unavailable": f"no host reference for workload {name}"}))
        return
    cores, threads = host_threads()
    h = HOST_WORKLOADS[name]
    rows_mode = name in ROWS_WORKLOADS or args.sharded
    x = host_inputs(name, args.seed)
    for _ in range(args.warmup):
        host_step(name, x)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        host_step(name, x)
        times.append(time.perf_counter() - t0)
    sec = float(np.mean(times))
    value = h["sample_B"] * h["T"] / sec
    sample = host_sample_desc(name)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong" if rows_mode else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": run_config(name, world, rows_mode),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "threads": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "host": {"os_cpu_count": cores, "blas_threads": threads}}
    print(json.dumps(line), flush=True)


def cpu_baseline(name, seed, budget_s):
    """The host path on a bounded sample of workload ``name`` (rank 0, N=1)."""
    cores, threads = host_threads()
    h = HOST_WORKLOADS[name]
    x = host_inputs(name, seed)
    host_step(name, x)   # warm-up
    times = []
    t0 = time.perf_counter()
    while not times or (time.perf_counter() - t0 < budget_s and len(times) < 20):
        s = time.perf_counter()
        host_step(name, x)
        times.append(time.perf_counter() - s)
    sec = float(np.mean(times))
    return {"value": h["sample_B"] * h["T"] / sec, "unit": "tokens/s", "cores": cores, "threads": threads,
            "kind": "port", "sample": f"{len(times)} steps, each a " + host_sample_desc(name),
            "sec_per_step": sec}


# ======================================================================
# Device workloads
# ======================================================================
def build_device_workload(w, device, seed):
    """Seeded synthetic inputs of a data-parallel (replicated pool) workload,
    generated on the device (the small pool is 9.1 GB)."""
    import torch
    from matrix_b200.assembly import compute_key_cache
    cfg = w.cfg
    g = torch.Generator(device=device).manual_seed(seed)
    d, D, N, S, dk, C = cfg.d_A, cfg.D, cfg.N, cfg.S, cfg.d_k, cfg.C
    bf = torch.bfloat16
    pool = torch.empty((N, D), dtype=bf, device=device)
    for i in range(0, N, 16384):
        pool[i:i + 16384].normal_(0.0, d ** -0.5, generator=g)
    key_proj = (torch.randn((S, D, dk), generator=g, device=device) * D ** -0.5).to(bf)
    keys = compute_key_cache(pool, key_proj)        # once per window in training (outside the step)
    off = torch.arange(C + 1, dtype=torch.int64, device=device) * (N // C)
    rows = off[:-1] + torch.randint(0, N // C, (C,), generator=g, device=device)
    return dict(
        pool=pool, key_proj=key_proj, keys=keys, list_offsets=off, centroids=keys[:, rows, :].contiguous(),
        W_Q=torch.randn((S, dk, d), generator=g, device=device) * d ** -0.5,
        aspect_weights=torch.zeros(S, device=device), tau=torch.zeros(1, device=device),
        W_base=torch.randn((d, d), generator=g, device=device) * 0.01,
        b_base=torch.zeros(d, device=device),
        gamma=torch.full((1,), cfg.gamma_init, device=device),
        lam=torch.full((1,), w.lambda_val, device=device),
        h_A=torch.randn((w.batch, w.seq, d), generator=g, device=device).to(bf),
        g_hmid=(torch.randn((w.batch, w.seq, d), generator=g, device=device) * 0.1).to(bf),
        g_W=torch.randn((w.batch, d, d), generator=g, device=device) * 1e-3,
    )


class Step:
    """One data-parallel step on device-resident inputs through the C ABI."""

    def __init__(self, w, t, group):
        import torch
        from matrix_b200 import _lib
        self.w, self.t, self.group = w, t, group
        self.lib = _lib.load()
        self.z = torch.empty((w.batch, w.cfg.d_A), dtype=torch.float32, device=t["h_A"].device)
        self.comm_events = None

    def __call__(self, h_A=None, g_hmid=None, g_W=None):
        import torch
        from matrix_b200 import _lib, runtime
        from matrix_b200.assembly import assemble_backward, assemble_forward
        from matrix_b200.retrieval import retrieve
        w, t, cfg = self.w, self.t, self.w.cfg
        h_A = t["h_A"] if h_A is None else h_A
        g_hmid = t["g_hmid"] if g_hmid is None else g_hmid
        g_W = t["g_W"] if g_W is None else g_W
        dev = h_A.device
        _lib.check(self.lib.dwa_sequence_mean(runtime.stream_of(dev), w.batch, w.seq, cfg.d_A, 1,
                                              runtime.ptr(h_A), runtime.ptr(self.z)), "dwa_sequence_mean")
        alphas, indices, soft_full = retrieve(
            self.z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], t["keys"], t["lam"],
            w.is_warmup, k=cfg.k_max, m=cfg.m, T=cfg.T, list_offsets=t["list_offsets"],
            max_list=cfg.N // cfg.C, want_soft_full=w.soft_full)
        h_mid, W, W_act = assemble_forward(t["pool"], alphas, h_A, t["W_base"], t["b_base"],
                                           t["gamma"], cfg.d_B, cfg.r, cfg.d_A, row_index=indices)
        out = dict(alphas=alphas, indices=indices, soft_full=soft_full, h_mid=h_mid, W=W)
        if w.backward:
            g = assemble_backward(t["pool"], alphas, h_A, W_act, t["gamma"], g_hmid, g_W,
                                  cfg.d_B, cfg.r, cfg.d_A, row_index=indices)
            out.update(zip(("g_rows", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), g))
            if self.group is not None:
                import torch.distributed as dist
                flat = torch.cat([out["g_W_base"].reshape(-1), out["g_b_base"], out["g_gamma"]])
                with comm_timer(self.comm_events, "param_allreduce"):
                    dist.all_reduce(flat, group=self.group)
                out["g_params"] = flat
        return out


class comm_timer:
    """Event pair around one collective (recorded into a graph capture as
    external event nodes) when ``events`` maps its name to a pair."""

    def __init__(self, events, name):
        self.pair = events.get(name) if events else None

    def __enter__(self):
        if self.pair:
            self.pair[0].record()

    def __exit__(self, *exc):
        if self.pair:
            self.pair[1].record()
        return False


def build_sharded_workload(w, device, rank, world, group, seed, emulate=0):
    """Rank ``rank``'s part of a row-sharded pool: the rows ``[lo, hi)`` (whole
    lists, balanced by rows) and their keys; the replicated parameters (same
    seed on every rank, centroids = key rows at random indices, combined by an
    all-reduce); this rank's ``w.batch / world`` sequences.  ``emulate = P``
    (one process): the rank of P with the most rows, whose sequences' queries
    are joined by the other ranks' (all ``w.batch`` sequences are generated for
    the query means) and whose centroids of lists held elsewhere are random
    vectors of the keys' scale."""
    shares = emulate if emulate else world
    import torch
    from matrix_b200.assembly import compute_key_cache
    from matrix_b200.sharded import shard_rows
    from matrix_b200.synthetic import zipf_list_offsets
    cfg = w.cfg
    d, D, N, S, dk, C = cfg.d_A, cfg.D, cfg.N, cfg.S, cfg.d_k, cfg.C
    if w.batch % shares:
        raise ValueError("the global batch must split evenly over the ranks")
    rng = np.random.default_rng(seed)
    off_np = (zipf_list_offsets(N, C, w.zipf, rng) if w.zipf else np.arange(C + 1, dtype=np.int64) * (N // C))
    bounds = shard_rows(off_np, shares)
    if emulate:   # the rank with the most rows, which sets the step time of the job
        rank = int(np.argmax([h - l for l, h in bounds]))
    lo, hi = bounds[rank]
    bf = torch.bfloat16
    g_rows = torch.Generator(device=device).manual_seed(seed + 1 + rank)     # this rank's pool rows
    pool = torch.empty((hi - lo, D), dtype=bf, device=device)
    for i in range(0, hi - lo, 16384):
        pool[i:i + 16384].normal_(0.0, d ** -0.5, generator=g_rows)
    g = torch.Generator(device=device).manual_seed(seed)                    # replicated parameters
    key_proj = (torch.randn((S, D, dk), generator=g, device=device) * D ** -0.5).to(bf)
    keys = compute_key_cache(pool, key_proj)
    del key_proj
    sizes = np.diff(off_np)
    rows_c = off_np[:-1] + (rng.random(C) * sizes).astype(np.int64)
    cent = torch.zeros((S, C, dk), device=device)
    mine = np.nonzero((rows_c >= lo) & (rows_c < hi))[0]
    if mine.size:
        cent[:, torch.from_numpy(mine).to(device)] = keys[:, torch.from_numpy(rows_c[mine] - lo).to(device)]
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(cent, group=group)
    if emulate:
        others = np.nonzero((rows_c < lo) | (rows_c >= hi))[0]
        if others.size:
            scale = float(keys.std())
            cent[:, torch.from_numpy(others).to(device)] = torch.randn(
                (S, others.size, dk), generator=torch.Generator(device=device).manual_seed(seed + 3),
                device=device) * scale
    Bp = w.batch // shares
    gs = torch.Generator(device=device).manual_seed(seed + 7919 * (rank + 1))  # this rank's sequences
    t = dict(
        pool=pool, keys=keys, row_lo=lo, row_hi=hi, bounds=bounds, list_offsets=torch.from_numpy(off_np).to(device),
        max_list=int(sizes.max()), centroids=cent.contiguous(),
        W_Q=torch.randn((S, dk, d), generator=g, device=device) * d ** -0.5,
        aspect_weights=torch.zeros(S, device=device), tau=torch.zeros(1, device=device),
        W_base=torch.randn((d, d), generator=g, device=device) * 0.01,
        b_base=torch.zeros(d, device=device),
        gamma=torch.full((1,), cfg.gamma_init, device=device),
        lam=torch.full((1,), w.lambda_val, device=device),
        h_A=torch.randn((Bp, w.seq, d), generator=gs, device=device).to(bf),
    )
    if emulate:   # the other ranks' sequences, for the queries only
        t["h_A_rest"] = torch.randn((w.batch - Bp, w.seq, d), generator=gs, device=device).to(bf)
        t["rank"] = rank
    if w.backward:
        t["g_hmid"] = (torch.randn((Bp, w.seq, d), generator=gs, device=device) * 0.1).to(bf)
        t["g_W"] = torch.randn((Bp, d, d), generator=gs, device=device) * 1e-3
        t["g_pool"] = torch.zeros((hi - lo, D), dtype=bf, device=device)
    return t


class ShardedStep:
    """One step of a row-sharded pool on this rank: the sequence means of its
    sequences, one all-gather of z, row-sharded retrieval (local top-k, one
    all-gather of the summaries, merge), the winning rows of its sequences read
    from the ranks that hold them (peer loads; with one rank the assembly reads
    them from the pool by index), their assembly and, with the backward, the
    rows' gradients returned to their owners and the parameter gradients
    all-reduced."""

    def __init__(self, w, t, group, rank, world, emulate=0):
        import torch
        from matrix_b200 import _lib
        from matrix_b200.peer import PeerPool
        self.w, self.t, self.group, self.rank, self.world = w, t, group, rank, world
        self.emulate = emulate
        self.apply_only = w.seq == 1 and not w.backward
        self.lib = _lib.load()
        self.comm_events = None
        dev = t["h_A"].device
        Bp = w.batch // (emulate or world)
        if emulate:
            rank = t["rank"]
            self.z_rest = torch.empty((w.batch - Bp, w.cfg.d_A), dtype=torch.float32, device=dev)
        self.b0, self.b1 = rank * Bp, (rank + 1) * Bp
        self.z_local = torch.empty((Bp, w.cfg.d_A), dtype=torch.float32, device=dev)
        self.z = torch.empty((w.batch, w.cfg.d_A), dtype=torch.float32, device=dev)
        self.peers = None
        if emulate:
            self.peers = PeerPool.from_shards([t["pool"]], [t["row_lo"], t["row_hi"]])
        elif world > 1:
            bounds = [t["bounds"][0][0]] + [h for _, h in t["bounds"]]
            self.peers = PeerPool(t["pool"], bounds, group)
        self.exchange = None
        if w.backward and world > 1 and not emulate:
            from matrix_b200.pool_grad import PoolGradExchange
            self.exchange = PoolGradExchange(bounds, Bp * w.cfg.k_max, w.cfg.D, dev, group)
        # the query means through peer-mapped buffers (NCCL all-gather if off)
        self.z_gather = None
        if world > 1 and not emulate:
            from matrix_b200.sharded import peer_gather
            self.z_gather = peer_gather(self.z_local.numel() * 4, dev, group)

    def __call__(self, h_A=None):
        from matrix_b200 import _lib, runtime
        from matrix_b200.assembly import assemble_backward, assemble_forward
        from matrix_b200.pool_grad import scatter_pool_grad_gathered
        from matrix_b200.sharded import RowShard, sharded_retrieve
        w, t, cfg = self.w, self.t, self.w.cfg
        h_A = t["h_A"] if h_A is None else h_A
        dev = h_A.device
        _lib.check(self.lib.dwa_sequence_mean(runtime.stream_of(dev), self.z_local.shape[0], w.seq, cfg.d_A, 1,
                                              runtime.ptr(h_A), runtime.ptr(self.z_local)), "dwa_sequence_mean")
        if self.world > 1:
            import torch.distributed as dist
            with comm_timer(self.comm_events, "allgather_z"):
                if self.z_gather is not None:
                    self.z_gather(self.z_local, self.z)
                else:
                    dist.all_gather_into_tensor(self.z, self.z_local, group=self.group)
            z = self.z
        elif self.emulate:
            # the other ranks' query means, in place of the all-gather
            Bq = w.batch - self.z_local.shape[0]
            _lib.check(self.lib.dwa_sequence_mean(runtime.stream_of(dev), Bq, w.seq, cfg.d_A, 1,
                                                  runtime.ptr(t["h_A_rest"]), runtime.ptr(self.z_rest)),
                       "dwa_sequence_mean")
            self.z[: self.b0].copy_(self.z_rest[: self.b0])
            self.z[self.b0: self.b1].copy_(self.z_local)
            self.z[self.b1:].copy_(self.z_rest[self.b0:])
            z = self.z
        else:
            z = self.z_local
        with comm_timer(self.comm_events, "retrieve_sharded"):
            if self.world == 1 and not self.emulate:     # every row here: the single-device call
                from matrix_b200.retrieval import retrieve
                alphas, indices, soft = retrieve(
                    z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], t["keys"], t["lam"], w.is_warmup,
                    k=cfg.k_max, m=cfg.m, T=cfg.T, list_offsets=t["list_offsets"], max_list=t["max_list"],
                    want_soft_full=w.soft_full)
            else:
                alphas, indices, soft = sharded_retrieve(
                    z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], t["keys"], t["list_offsets"],
                    t["lam"], w.is_warmup, RowShard(t["row_lo"], t["row_hi"], cfg.N, self.group), k=cfg.k_max,
                    m=cfg.m, T=cfg.T, max_list=t["max_list"], want_soft_full=w.soft_full)
        idx_mine = indices[self.b0:self.b1]
        al_mine = alphas[self.b0:self.b1]
        if self.peers is not None:
            rows, row_index = self.peers.gather(idx_mine), None
        else:
            rows, row_index = t["pool"], idx_mine
        if self.apply_only:     # generation: h_mid only, W never formed (dwa_assemble_apply)
            from matrix_b200.assembly import assemble_apply
            h_mid, W = assemble_apply(rows, al_mine, h_A, t["W_base"], t["b_base"], t["gamma"], cfg.d_B, cfg.r,
                                      cfg.d_A, row_index=row_index), None
        else:
            h_mid, W, W_act = assemble_forward(rows, al_mine, h_A, t["W_base"], t["b_base"], t["gamma"],
                                               cfg.d_B, cfg.r, cfg.d_A, row_index=row_index)
        out = dict(alphas=alphas, indices=indices, soft_full=soft, h_mid=h_mid, W=W,
                   rows=rows if row_index is None else None)
        if w.backward:
            g = assemble_backward(rows, al_mine, h_A, W_act, t["gamma"], t["g_hmid"], t["g_W"],
                                  cfg.d_B, cfg.r, cfg.d_A, row_index=row_index)
            out.update(zip(("g_rows", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), g))
            with comm_timer(self.comm_events, "rowgrad_exchange"):
                if self.exchange is not None:     # bf16 rows stored into their owners' receive areas
                    self.exchange(g[0], idx_mine, t["g_pool"])
                else:
                    scatter_pool_grad_gathered(g[0], idx_mine, t["g_pool"], row_lo=t["row_lo"], n_global=cfg.N,
                                               group=None)
            if self.world > 1:
                import torch
                import torch.distributed as dist
                flat = torch.cat([out["g_W_base"].reshape(-1), out["g_b_base"], out["g_gamma"]])
                with comm_timer(self.comm_events, "param_allreduce"):
                    dist.all_reduce(flat, group=self.group)
                out["g_params"] = flat
        return out


# ======================================================================
# Timing
# ======================================================================
def kernel_work(w, name, n_rows=None, seqs=None):
    """Algorithmic bytes (HBM-bound kernels) or flops (tensor kernels) of one
    launch of `name` on workload w; returns (bound, amount).  A rank of a
    row-sharded pool scores ``n_rows`` rows for all ``w.batch`` queries and
    assembles ``seqs`` sequences."""
    c = w.cfg
    B, T, d, k, r, S, dk = w.batch, w.seq, c.d_A, c.k_max, c.r, c.S, c.d_k
    N = c.N if n_rows is None else n_rows
    Ba = B if seqs is None else seqs
    kr = k * r
    table = {
        "full_scores": ("hbm", 4 * (S * N * dk + B * N)),
        "fine": ("hbm", 4 * (B * S * min(c.m, c.C) * (c.N // c.C) * dk)),
        "softmax_apply": ("hbm", 8 * B * N),
        "prep_factors": ("hbm", Ba * k * (d * r + r * d) * 2 * 2),
        "gemm_W": ("tensor", 2 * Ba * d * d * kr),
        "gemm_apply": ("tensor", 2 * Ba * T * d * d),
        "gemm_G": ("tensor", 2 * Ba * T * d * d),
        "gemm_gh": ("tensor", 2 * Ba * T * d * d),
        "gemm_P": ("tensor", 2 * Ba * d * d * kr),
        "gemm_Q": ("tensor", 2 * Ba * d * d * kr),
        "gather_rows": ("hbm", 2 * Ba * k * c.D * (2 if c.bf16_pool else 4)),
        # h_mid-only apply: the V part, then the U and b parts of every winning row
        "factored_hv": ("hbm", Ba * k * r * d * 2),
        "factored_out": ("hbm", Ba * k * (d * r + d) * 2),
    }
    return table.get(name, ("hbm", None))


def profiled_traffic(kernel, n_rows, queries):
    """DRAM bytes (read + write) per launch of `kernel`, from the `traffic:`
    lines of the ncu summaries under profiles/ (the one whose query count
    matches, else any): a summary captured on a smaller case is scaled by the
    key rows it read (keys and s_full writes both grow with the rows)."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    best = None
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".txt"):
            continue
        with open(os.path.join(d, fn)) as f:
            for line in f:
                if not line.startswith("traffic:"):
                    continue
                kv = dict(tok.split("=", 1) for tok in line.split()[1:] if "=" in tok)
                if kv.get("kernel") != kernel:
                    continue
                if best is None or int(kv.get("queries", -1)) == queries:
                    best = kv
    if best is None:
        return None
    q0 = int(best["queries"])
    bytes0 = int(best["dram_read_bytes"]) + int(best["dram_write_bytes"])
    rows0 = float(best["rows"])
    # per row: the key stream (fixed) plus q s_full floats written
    per_row = bytes0 / rows0
    return int(per_row * n_rows + 4 * n_rows * (queries - q0))


KERNELS = ["seq_mean", "query", "query_norm", "coarse", "topm", "full_scores", "fine", "select",
           "softmax_stats",
           "softmax_apply", "prep_factors", "prep_bias", "gemm_W", "gemm_apply", "gemm_G",
           "gemm_gh", "gemm_P", "gemm_Q", "colsum", "finalize", "bias_grad", "merge", "gather_rows",
           "factored_hv", "base_rows", "cast_w_base", "gemm_base", "factored_out", "factored_combine", "probe_lists",
           "scatter_sort", "scatter_add", "grad_send"]
COMM = ["allgather_z", "retrieve_sharded", "rowgrad_exchange", "param_allreduce"]


def C_ptr(event):
    import ctypes
    return ctypes.c_void_p(event.cuda_event)


def capture(step, n_pre=1):
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(n_pre):
            step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    return g


def profile_kernels(step, flush, group, n=5):
    """Per-kernel device time (ms) of one step, additive: the step is captured
    with serialised launches (no programmatic dependent launch, the calls'
    concurrent lanes on one stream) and an event pair around every library
    kernel and every collective; averaged over ``n`` replays.  Returns
    (durations, starts relative to the step's first kernel, serialised step
    ms)."""
    import torch
    from matrix_b200 import _lib
    lib = _lib.load()
    mk = lambda: (torch.cuda.Event(enable_timing=True, external=True),  # noqa: E731
                  torch.cuda.Event(enable_timing=True, external=True))
    ev = {k: mk() for k in KERNELS}
    comm = {k: mk() for k in COMM}
    for a, b in list(ev.values()) + list(comm.values()):   # torch creates the CUDA event on first record
        a.record(); b.record()
    torch.cuda.synchronize()
    for k, (a, b) in ev.items():
        lib.dwa_profile_kernel(k.encode(), C_ptr(a), C_ptr(b))
    lib.dwa_profile_serialize(1)
    step.comm_events = comm
    try:
        g = capture(step)
    finally:
        step.comm_events = None
        lib.dwa_profile_serialize(0)
        lib.dwa_profile_clear()
    whole = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    acc = {k: [] for k in KERNELS + COMM}
    start = {k: [] for k in KERNELS + COMM}
    total = []
    for _ in range(n):
        flush()
        sync_ranks(group)
        whole[0].record()
        g.replay()
        whole[1].record()
        torch.cuda.synchronize()
        total.append(whole[0].elapsed_time(whole[1]))
        for k, (a, b) in list(ev.items()) + list(comm.items()):
            t0 = whole[0].elapsed_time(a)
            if t0 >= 0.0:
                acc[k].append(a.elapsed_time(b))
                start[k].append(t0)
    del g
    dur = {k: float(np.mean(v)) for k, v in acc.items() if v}
    return dur, {k: float(np.mean(start[k])) for k in dur}, float(np.mean(total))


def split_breakdown(dur):
    """(library kernels, collectives / wrapped phases) of a profile_kernels
    result; the kernels alone add up to the serialised step on one GPU."""
    return ({k: v for k, v in dur.items() if k in KERNELS}, {k: v for k, v in dur.items() if k in COMM})


def sync_ranks(group):
    import torch
    torch.cuda.synchronize()
    if group is not None:
        import torch.distributed as dist
        dist.barrier(group=group)
        torch.cuda.synchronize()


class ClockSampler:
    """nvidia-smi samples of the SM clock, power and throttle reasons of the
    given GPUs (by UUID), 200 ms apart, while the timed region runs."""
    QUERY = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = {u.lower().replace("gpu-", "") for u in uuids}
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9 or f[0].lower().replace("gpu-", "") not in self.uuids:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        out = {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm), "gpus": len(self.uuids)}
        if power:
            out["power_w_max"] = float(max(power))
        return out


def device_uuids(dev, group):
    import torch
    u = str(torch.cuda.get_device_properties(dev).uuid)
    if group is None:
        return [u]
    import torch.distributed as dist
    every = [None] * dist.get_world_size(group)
    dist.all_gather_object(every, u, group=group)
    return every


def measure(step, flush, group, dev, steps, warmup, rank, sample_clocks=True):
    """Launch count, additive kernel breakdown, then the timed graph replays:
    ``steps`` replays after ``warmup``, each after an L2 flush and a barrier,
    CUDA events around each replay, per-step maximum over ranks; the dominant
    kernel re-timed live inside the timed replays (external event nodes)."""
    import torch
    from matrix_b200 import _lib
    lib = _lib.load()
    step()                       # first call: workspaces, kernel attributes
    torch.cuda.synchronize()
    c0 = _lib.launch_counters()[0]
    step()
    torch.cuda.synchronize()
    launches = _lib.launch_counters()[0] - c0
    breakdown, kstarts, serial_ms = profile_kernels(step, flush, group)
    dominant = max((k for k in breakdown if k in KERNELS), key=breakdown.get)

    ka = torch.cuda.Event(enable_timing=True, external=True)
    kb = torch.cuda.Event(enable_timing=True, external=True)
    ka.record(); kb.record()
    torch.cuda.synchronize()
    lib.dwa_profile_kernel(dominant.encode(), C_ptr(ka), C_ptr(kb))
    try:
        graph = capture(step, n_pre=2)
    finally:
        lib.dwa_profile_clear()
    for _ in range(max(warmup, 3)):
        flush()
        graph.replay()
    uuids = device_uuids(dev, group)
    sampler = ClockSampler(uuids) if (rank == 0 and sample_clocks) else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    kern_ms = []
    sync_ranks(group)
    for i in range(steps):
        flush()
        sync_ranks(group)
        starts[i].record()
        graph.replay()
        stops[i].record()
        stops[i].synchronize()
        kern_ms.append(ka.elapsed_time(kb))
    sync_ranks(group)
    clocks = sampler.stop() if sampler else None
    per_step = torch.tensor([a.elapsed_time(b) for a, b in zip(starts, stops)], device=dev, dtype=torch.float64)
    mine = float(per_step.mean().item())
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(per_step, op=dist.ReduceOp.MAX, group=group)
    del graph
    return dict(ms_per_step=float(per_step.sum().item()) / steps, rank_ms_per_step=mine, launches=int(launches),
                breakdown=breakdown, starts=kstarts, serial_ms=serial_ms, dominant=dominant,
                kern_ms=float(np.mean(kern_ms)), clocks=clocks)


def roofline(w, m, peaks, peak_src, n_rows=None, seqs=None, queries=None):
    bound, work = kernel_work(w, m["dominant"], n_rows=n_rows, seqs=seqs)
    if work is None:
        return None
    kms = m["kern_ms"]
    if bound == "hbm":
        ach, peak, unit = work / (kms / 1e3) / 1e9, float(peaks["hbm_gbs"]), "GB/s"
    else:
        ach, peak, unit = work / (kms / 1e3) / 1e12, float(peaks["bf16_tflops"]), "TFLOP/s"
    traffic = None
    if m["dominant"] == "full_scores":
        traffic = profiled_traffic("full_scores", n_rows if n_rows is not None else w.cfg.N,
                                   queries if queries is not None else w.batch)
    return {"kernel": m["dominant"], "bound": bound, "achieved": ach, "peak": peak, "unit": unit,
            "frac": ach / peak, "traffic": traffic, "peak_source": peak_src,
            "algorithmic_per_launch": work, "launch_ms": kms,
            "timed_in": "graph replay of the timed steps (external event nodes)"}


# ======================================================================
# Parity of the row-sharded step
# ======================================================================
def rows_parity(w, t, step, group, rank, world):
    """The sharded retrieval against ``dwa_retrieve`` on one device over the
    all-gathered key cache (same z): indices equal, alphas and soft_full within
    rtol 1e-5; and, with several ranks, each rank's peer-read rows against the
    reference's masked-psum gather (model.py:16-47: every rank contributes the
    rows it holds, zeros elsewhere, summed over the ranks).  Runs after the
    timing, outside the timed region."""
    import torch
    from matrix_b200.retrieval import retrieve
    cfg = w.cfg
    dev = t["keys"].device
    out = step()
    torch.cuda.synchronize()
    S, n_loc, dk = t["keys"].shape
    z = step.z if (world > 1 or step.emulate) else step.z_local
    if world > 1:
        import torch.distributed as dist
        n_max = max(h - l for l, h in t["bounds"])
        pad = torch.zeros((S, n_max, dk), device=dev)
        pad[:, :n_loc] = t["keys"]
        allk = torch.empty((world, S, n_max, dk), device=dev)
        dist.all_gather_into_tensor(allk, pad, group=group)
        keys = torch.cat([allk[p, :, :h - l] for p, (l, h) in enumerate(t["bounds"])], dim=1).contiguous()
        del allk, pad
        sf = None
        if out["soft_full"] is not None:
            spad = torch.zeros((w.batch, n_max), device=dev)
            spad[:, :n_loc] = out["soft_full"]
            alls = torch.empty((world, w.batch, n_max), device=dev)
            dist.all_gather_into_tensor(alls, spad, group=group)
            sf = torch.cat([alls[p, :, :h - l] for p, (l, h) in enumerate(t["bounds"])], dim=1)
            del alls, spad
    else:
        keys, sf = t["keys"], out["soft_full"]
    a1, i1, s1 = retrieve(z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], keys, t["lam"], w.is_warmup,
                          k=cfg.k_max, m=cfg.m, T=cfg.T, list_offsets=t["list_offsets"], max_list=t["max_list"],
                          want_soft_full=w.soft_full)
    res = {"indices_equal": bool(torch.equal(i1, out["indices"])),
           "alphas_max_rel_err": float(((a1 - out["alphas"]).abs() / a1.abs().clamp_min(1e-30)).max().item())}
    if s1 is not None and sf is not None:
        res["soft_full_max_err_rel_to_max"] = float(((s1 - sf).abs().max() / s1.abs().max()).item())
    del keys
    if world > 1:
        import torch.distributed as dist
        idx = out["indices"].reshape(-1).long()
        lo, hi = t["row_lo"], t["row_hi"]
        mask = (idx >= lo) & (idx < hi)
        full = torch.zeros((idx.numel(), cfg.D), dtype=t["pool"].dtype, device=dev)
        full[mask] = t["pool"][idx[mask] - lo]
        dist.all_reduce(full, group=group)
        Bp = w.batch // world
        mine = full.reshape(w.batch, cfg.k_max, cfg.D)[rank * Bp:(rank + 1) * Bp]
        res["rows_equal"] = bool(torch.equal(mine, out["rows"]))
        del full
        flags = torch.tensor([float(res["indices_equal"]), float(res["rows_equal"])], device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN, group=group)
        errs = torch.tensor([res["alphas_max_rel_err"], res.get("soft_full_max_err_rel_to_max", 0.0)], device=dev)
        dist.all_reduce(errs, op=dist.ReduceOp.MAX, group=group)
        res.update(indices_equal=bool(flags[0] > 0), rows_equal=bool(flags[1] > 0),
                   alphas_max_rel_err=float(errs[0]), soft_full_max_err_rel_to_max=float(errs[1]),
                   ranks_checked=world)
    else:
        res["rows_equal"] = None
    res["ok"] = bool(res["indices_equal"] and res["alphas_max_rel_err"] <= 1e-5
                     and res.get("soft_full_max_err_rel_to_max", 0.0) <= 1e-5
                     and res["rows_equal"] is not False)
    res["against"] = ("dwa_retrieve on one device over the all-gathered key cache; rows: the masked-psum "
                      "gather of the reference's model-sharded path")
    torch.cuda.synchronize()
    return res


# ======================================================================
# End to end through the public API with pinned host buffers
# ======================================================================
def e2e_pipeline(step_fn, host_inputs_, result_keys, n, group, dev):
    """A training input pipeline: step i+1's inputs go up on a copy stream while
    step i computes and step i-1's results come down on another; device inputs
    and pinned host outputs are double-buffered, and the step on each input
    buffer is a CUDA graph (captured once, as a serving loop would), so the
    host issues one replay per step.  Every step's host->device and
    device->host copies are inside the timed region.  Returns (ms per step,
    max over ranks; h2d bytes; d2h bytes)."""
    import torch
    dev_bufs = [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host_inputs_] for _ in range(2)]
    for bufs in dev_bufs:
        for b, h in zip(bufs, host_inputs_):
            b.copy_(h)
    graphs, outs = [], []
    for bufs in dev_bufs:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step_fn(*bufs)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            o = step_fn(*bufs)
        graphs.append(g)
        outs.append(o)
    out = outs[0]
    torch.cuda.synchronize()
    pins = [{k: torch.empty(out[k].shape, dtype=out[k].dtype).pin_memory() for k in result_keys} for _ in range(2)]
    h2d = sum(h.nbytes for h in host_inputs_)
    d2h = sum(v.nbytes for v in pins[0].values())
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    main = torch.cuda.current_stream()
    ev_in = [torch.cuda.Event() for _ in range(n)]
    ev_used = [torch.cuda.Event() for _ in range(n)]
    ev_out = [torch.cuda.Event() for _ in range(n)]
    t_start, t_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_ranks(group)
    ring = [None, None]     # step outputs alive until their copy to the host is done
    t_start.record(main)
    s_in.wait_event(t_start)
    for i in range(n):
        bufs = dev_bufs[i % 2]
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_used[i - 2])      # step i-2 has read this buffer
            for b, h in zip(bufs, host_inputs_):
                b.copy_(h, non_blocking=True)
            ev_in[i].record(s_in)
        main.wait_event(ev_in[i])
        if i >= 2:
            main.wait_event(ev_out[i - 2])           # step i-2's outputs reached the host
            ring[i % 2] = None
        graphs[i % 2].replay()
        out = outs[i % 2]
        ev_used[i].record(main)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_used[i])
            for k in result_keys:
                pins[i % 2][k].copy_(out[k], non_blocking=True)
            ev_out[i].record(s_out)
        ring[i % 2] = out
    main.wait_event(ev_out[n - 1])
    t_stop.record(main)
    t_stop.synchronize()
    del graphs, outs, ring
    e_ms = torch.tensor([t_start.elapsed_time(t_stop) / n], device=dev, dtype=torch.float64)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX, group=group)
    return float(e_ms.item()), int(h2d), int(d2h)


# ======================================================================
# Extras at N=1 (small workload)
# ======================================================================
def time_key_cache(t, flush, peaks, reps=3):
    """``compute_key_cache`` on the workload's pool (once per training window,
    not part of the step), timed with CUDA events after a flush, against its
    HBM and bf16 rooflines; cuBLAS's bf16 GEMM of the same product
    (``pool @ key_proj`` into ``[N, S*d_k]``, no re-layout) as a library reference."""
    import torch
    from matrix_b200.assembly import compute_key_cache
    pool, kp = t["pool"], t["key_proj"]
    N, D = pool.shape
    S, _, dk = kp.shape
    kp2 = kp.permute(1, 0, 2).reshape(D, S * dk).contiguous()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        ms = []
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ms.append(a.elapsed_time(b))
        return float(min(ms))

    ours = timed(lambda: compute_key_cache(pool, kp))
    lib = timed(lambda: torch.matmul(pool, kp2))
    flops = 2.0 * N * D * S * dk
    hbm = float(N * D * 2 + S * N * dk * 4 + S * D * dk * 2)
    t_hbm = hbm / (float(peaks["hbm_gbs"]) * 1e9) * 1e3
    t_tc = flops / (float(peaks["bf16_tflops"]) * 1e12) * 1e3
    return {"ms": ours, "tflops": flops / (ours * 1e-3) / 1e12, "hbm_gbs": hbm / (ours * 1e-3) / 1e9,
            "roofline_ms": max(t_hbm, t_tc), "frac": max(t_hbm, t_tc) / ours,
            "bound": "hbm" if t_hbm >= t_tc else "tensor", "algorithmic_bytes": hbm, "flops": flops,
            "cublas_gemm_ms": lib, "shape": f"pool [{N}, {D}] bf16 x key_proj [{S}, {D}, {dk}] bf16"}


def time_training_extras(w, t, flush, peaks, reps=5):
    """The retrieval VJP (alphas' cotangent alone, with soft_full's, with the
    key-cache gradient; key pass against its HBM roofline) and the aux losses,
    on the small workload's inputs, timed with CUDA events after a flush (best
    of ``reps``).  The cotangents are seeded synthetic values."""
    import torch
    from matrix_b200 import _lib
    from matrix_b200.losses import aux_losses_and_grads
    from matrix_b200.retrieval import retrieve, retrieve_backward
    lib = _lib.load()
    cfg = w.cfg
    g = torch.Generator(device=t["keys"].device).manual_seed(7)
    z = t["h_A"].float().mean(dim=1)
    kw = dict(k=cfg.k_max, m=cfg.m, T=cfg.T, list_offsets=t["list_offsets"], max_list=cfg.N // cfg.C)
    args = (z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], t["keys"], t["lam"], w.is_warmup)
    alphas, indices, soft_full = retrieve(*args, **kw, want_soft_full=True)
    g_al = torch.randn(alphas.shape, generator=g, device=z.device)
    g_sf = torch.randn(soft_full.shape, generator=g, device=z.device)

    def timed(fn, name=None):
        fn()
        torch.cuda.synchronize()
        ms, kms = [], []
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        if name:
            for e in ev:
                e.record()
            torch.cuda.synchronize()
            lib.dwa_profile_kernel(name.encode(), C_ptr(ev[0]), C_ptr(ev[1]))
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ms.append(a.elapsed_time(b))
            if name:
                kms.append(ev[0].elapsed_time(ev[1]))
        if name:
            lib.dwa_profile_clear()
        return float(min(ms)), (float(min(kms)) if kms else None)

    def bwd(gs, keys):
        return retrieve_backward(*args, alphas, indices, soft_full, g_al, gs, **kw, want_key_grad=keys)

    probed_ms, _ = timed(lambda: bwd(None, False))
    full_ms, kp_ms = timed(lambda: bwd(g_sf, False), name="key_grad")
    keys_ms, kp_keys_ms = timed(lambda: bwd(g_sf, True), name="key_grad")
    S, N, dk = t["keys"].shape
    B = z.shape[0]
    kp_bytes = 4.0 * (S * N * dk + B * N)
    out = {"retrieve_bwd": {
        "alphas_only_ms": probed_ms, "alphas_and_soft_full_ms": full_ms, "with_key_grad_ms": keys_ms,
        "key_pass_with_key_grad_ms": kp_keys_ms,
        "key_pass": {"kernel": "key_grad", "ms": kp_ms, "algorithmic_bytes": kp_bytes,
                     "hbm_gbs": kp_bytes / (kp_ms * 1e-3) / 1e9 if kp_ms else None,
                     "frac": (kp_bytes / (kp_ms * 1e-3) / 1e9) / float(peaks["hbm_gbs"]) if kp_ms else None},
        "shape": f"B {B}, keys [{S}, {N}, {dk}] f32, {cfg.m} probes of {cfg.N // cfg.C} rows, top-k {cfg.k_max}"}}
    W = torch.randn((B, cfg.d_B, cfg.d_A), generator=g, device=z.device) * 0.01
    aux_ms, _ = timed(lambda: aux_losses_and_grads(alphas, indices, t["keys"], W, t["W_base"], soft_full))
    out["aux_losses"] = {"ms": aux_ms, "shape": f"B {B}, k {cfg.k_max}, N {N}, W [{B}, {cfg.d_B}, {cfg.d_A}] f32"}
    return out


# ======================================================================
# Decode sweep (manual mode)
# ======================================================================
def decode_sweep(args, w, dev, flush, peaks, peak_src):
    """The decode workload on one GPU holding one rank's share of 8: 2M/8 =
    262144 pool rows x 69632 (d 4096, bf16, 36.5 GB) with their keys and 256
    of the 2048 lists (1024 rows each).  A step is one token for B sequences:
    sequence mean (T = 1), dwa_retrieve over this GPU's rows (gate mode,
    nprobe 16, no soft_full) and dwa_assemble_apply (h_mid only, the winning
    rows read from the pool by index).  ``decode_profile``: the same step at
    batch 256, top-k 128 on its own small pool (for ncu).  Returns one
    JSON-ready dict."""
    import torch
    from matrix_b200 import _lib, runtime
    from matrix_b200.assembly import assemble_apply, compute_key_cache
    from matrix_b200.retrieval import retrieve
    c = w.cfg
    share = 8 if w.name == "decode" else 1
    shapes = [(B, k) for B in (1, 8, 64, 256) for k in (16, 128)] if w.name == "decode" else [(w.batch, c.k_max)]
    d, D, S, dk, r = c.d_A, c.D, c.S, c.d_k, c.r
    N, C = c.N // share, c.C // share
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(args.seed)
    pool = torch.empty((N, D), dtype=torch.bfloat16, device=dev)
    for i in range(0, N, 8192):
        pool[i:i + 8192].normal_(0.0, d ** -0.5, generator=g)
    key_proj = (torch.randn((S, D, dk), generator=g, device=dev) * D ** -0.5).to(torch.bfloat16)
    keys = compute_key_cache(pool, key_proj)
    del key_proj
    rows_c = (torch.arange(C, device=dev) * (N // C) +
              torch.randint(0, N // C, (C,), generator=g, device=dev))
    cent = keys[:, rows_c].contiguous()
    W_Q = torch.randn((S, dk, d), generator=g, device=dev) * d ** -0.5
    aw, tau = torch.zeros(S, device=dev), torch.zeros(1, device=dev)
    W_base = torch.randn((d, d), generator=g, device=dev) * 0.01
    b_base = torch.zeros(d, device=dev)
    gamma = torch.full((1,), c.gamma_init, device=dev)
    lam = torch.full((1,), 5.0, device=dev)
    points = []
    for B, k in shapes:
        h_A = torch.randn((B, 1, d), generator=g, device=dev).to(torch.bfloat16)
        z = torch.empty((B, d), dtype=torch.float32, device=dev)

        class _Step:
            comm_events = None

            def __call__(self):
                _lib.check(lib.dwa_sequence_mean(runtime.stream_of(dev), B, 1, d, 1, runtime.ptr(h_A),
                                                 runtime.ptr(z)), "dwa_sequence_mean")
                al, idx, _ = retrieve(z, W_Q, aw, tau, cent, keys, lam, False, k=k, m=c.m, T=c.T,
                                      want_soft_full=False)
                return assemble_apply(pool, al, h_A, W_base, b_base, gamma, d, r, d, row_index=idx)

        m = measure(_Step(), flush, None, dev, 20, args.warmup, 0, sample_clocks=False)
        runtime.raise_on_device_status()
        ms = m["ms_per_step"]
        pt = {"batch": B, "top_k": k, "ms_per_token_step": ms, "tokens_per_s": B / (ms / 1e3),
              "kernels_ms": split_breakdown(m["breakdown"])[0], "gpu_launches_per_step": m["launches"],
              "gathered_row_bytes": B * k * D * 2}
        for name, part in (("factored_hv", r * d), ("factored_out", d * r + d)):
            if m["breakdown"].get(name):
                gbs = B * k * part * 2 / (m["breakdown"][name] / 1e3) / 1e9
                pt[name + "_gbs"] = gbs
                pt[name + "_frac"] = gbs / float(peaks["hbm_gbs"])
        points.append(pt)
    big = points[-1]
    return {"metric": METRIC, "value": big["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
            "steps": 20, "warmup": max(args.warmup, 3), "ms_per_step": big["ms_per_token_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": w.name, "note": w.note,
                       "this_gpu": (f"one rank's share of {share}: " if share > 1 else "") +
                                   f"{N} pool rows x {D}, {C} lists, nprobe {c.m}",
                       "mode": "gate lambda=5.0, no soft_full, h_mid only (dwa_assemble_apply)",
                       "l2": L2_NOTE, "step": "CUDA graph: seq_mean + dwa_retrieve + dwa_assemble_apply",
                       "headline": "batch 256, top-k 128"},
            "peak_hbm_gbs": float(peaks["hbm_gbs"]), "peak_source": peak_src, "sweep": points}


# ======================================================================
# Main
# ======================================================================
def ncu_steps(step, flush, group, n):
    """Eager steps inside NVTX ranges 'dwa_step', for an ncu launch list
    filtered with --nvtx --nvtx-include 'dwa_step/'."""
    import torch
    step()
    sync_ranks(group)
    for _ in range(n):
        flush()
        sync_ranks(group)
        torch.cuda.nvtx.range_push("dwa_step")
        step()
        torch.cuda.nvtx.range_pop()
    sync_ranks(group)
    print(json.dumps({"ncu_steps": n}), flush=True)
    if group is not None:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def small_dp_line(args, w, dev, group, rank, world, flush, peaks, peak_src, full=True):
    """The data-parallel small workload (fwd + bwd): every rank its own batch
    against its own pool replica.  ``full``: also e2e, key cache, extras."""
    t = build_device_workload(w, dev, args.seed + rank)
    step = Step(w, t, group)
    m = measure(step, flush, group, dev, args.steps, args.warmup, rank, sample_clocks=full)
    tokens = w.batch * w.seq * world
    kern, comm = split_breakdown(m["breakdown"])
    res = {"value": tokens / (m["ms_per_step"] / 1e3), "ms_per_step": m["ms_per_step"],
           "roofline": roofline(w, m, peaks, peak_src), "kernels_ms": kern, "comm_ms": comm,
           "kernels_sum_ms": float(sum(kern.values())),
           "kernels_start_ms": m["starts"], "serialized_step_ms": m["serial_ms"],
           "gpu_launches": m["launches"] * args.steps, "clocks": m["clocks"]}
    if full and not args.no_e2e:
        from matrix_b200 import runtime  # noqa: F401
        ins = [t["h_A"].cpu().pin_memory(), t["g_hmid"].cpu().pin_memory(), t["g_W"].cpu().pin_memory()]
        keys = ["h_mid", "g_hA", "g_rows", "g_alpha", "g_W_base", "g_b_base", "g_gamma", "alphas", "indices"]
        ms, h2d, d2h = e2e_pipeline(lambda a, b, c: step(a, b, c), ins, keys, min(args.steps, 50), group, dev)
        res["e2e"] = {"value": tokens / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h, "ms_per_step": ms,
                      "mode": "copies overlapped with compute on two copy streams, double-buffered"}
    if world == 1 and full:
        if not args.no_key_cache:
            res["key_cache"] = time_key_cache(t, flush, peaks)
        if not args.no_extras:
            res.update(time_training_extras(w, t, flush, peaks))
    return res


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from matrix_b200.config import WORKLOADS
    w = WORKLOADS[args.workload]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        group = dist.group.WORLD

    flush_buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        # write 512 MB (> 126 MB L2), then read back 256 MB of it: the write
        # evicts the step's data, the read makes the flush's dirty lines be
        # written back here rather than inside the next timed step
        flush_buf.zero_()
        flush_sink.copy_(flush_buf[: flush_buf.numel() // 2].sum())

    peaks, peak_src = load_peaks()
    if w.name in ("decode", "decode_profile") and world == 1 and not args.sharded:
        print(json.dumps(decode_sweep(args, w, dev, flush, peaks, peak_src)), flush=True)
        return
    if w.name == "decode":
        # several GPUs: the whole 2M-row pool row-sharded over them, one token of
        # 256 sequences with top-k 128 (the sweep's headline point), no soft_full
        from matrix_b200.config import scaled
        w = scaled(w, batch=256, k_max=128, soft_full=False, name="decode")

    rows_mode = w.name in ROWS_WORKLOADS or w.name == "decode" or args.sharded or args.emulate_ranks
    if not rows_mode and args.ncu_steps:
        return ncu_steps(Step(w, build_device_workload(w, dev, args.seed + rank), group), flush, group,
                         args.ncu_steps)
    if not rows_mode:
        r = small_dp_line(args, w, dev, group, rank, world, flush, peaks, peak_src)
        line = {"metric": METRIC, "value": r.pop("value"), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r.pop("ms_per_step"),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": run_config(w.name, world, False, w=w)}
        line.update(r)
        if rank == 0 and world == 1 and not args.no_cpu_baseline and w.name in HOST_WORKLOADS:
            cb = cpu_baseline(w.name, args.seed, args.cpu_budget_s)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "threads", "kind", "sample")}
        if rank == 0:
            print(json.dumps(line), flush=True)
        if group is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---------------- row-sharded pool (the default) ----------------
    if args.emulate_ranks and world > 1:
        raise SystemExit("--emulate-ranks runs on one GPU")
    emulate = args.emulate_ranks
    t = build_sharded_workload(w, dev, rank, world, group, args.seed, emulate=emulate)
    step = ShardedStep(w, t, group, rank, world, emulate=emulate)
    if args.ncu_steps:
        return ncu_steps(step, flush, group, args.ncu_steps)
    m = measure(step, flush, group, dev, args.steps, args.warmup, rank)
    Bp = w.batch // (emulate or world)
    n_loc = t["row_hi"] - t["row_lo"]
    tokens = (Bp if emulate else w.batch) * w.seq
    value = tokens / (m["ms_per_step"] / 1e3)
    roof = roofline(w, m, peaks, peak_src, n_rows=n_loc, seqs=Bp, queries=w.batch)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": run_config(w.name, world, True, emulate, w=w),
            "value_per_gpu": value / (1 if emulate else world), "roofline": roof,
            "kernels_ms": split_breakdown(m["breakdown"])[0], "comm_ms": split_breakdown(m["breakdown"])[1],
            "kernels_sum_ms": float(sum(split_breakdown(m["breakdown"])[0].values())),
            "kernels_start_ms": m["starts"], "serialized_step_ms": m["serial_ms"],
            "gpu_launches": m["launches"] * args.steps, "clocks": m["clocks"],
            "rows_per_rank": n_loc, "seqs_per_rank": Bp}
    if group is not None:
        every = [None] * world
        dist.all_gather_object(every, {"ms_per_step": m["rank_ms_per_step"], "kernels_ms": m["breakdown"],
                                       "rows": n_loc}, group=group)
        line["per_rank"] = every
    if emulate:
        line["config"]["emulated"] = (
            f"rank {t['rank']} of {emulate} (the most rows): pool rows [{t['row_lo']}, {t['row_hi']}) of "
            f"{w.cfg.N} (whole lists), retrieval of all {w.batch} queries over them, assembly of its {Bp} "
            f"sequences; the all-gathers, the merge across ranks, peer reads and the row-gradient exchange are "
            f"not in it")
    if not args.no_parity and not emulate:
        line["parity"] = rows_parity(w, t, step, group, rank, world)
    if not args.no_e2e and not emulate and not w.backward:
        hA_h = t["h_A"].cpu().pin_memory()
        ms, h2d, d2h = e2e_pipeline(lambda a: step(a), [hA_h], ["h_mid", "alphas", "indices"],
                                    min(args.steps, 20), group, dev)
        line["e2e"] = {"value": tokens / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                       "d2h_bytes_per_step": d2h * world, "ms_per_step": ms,
                       "mode": "every rank copies its sequences' h_A up and their h_mid, alphas and indices "
                               "down each step (bytes summed over ranks); copies overlapped with compute on "
                               "two copy streams, double-buffered"}
    from matrix_b200 import runtime
    if emulate:
        # one rank alone: its merge sees only its own candidates (fewer than k
        # for some queries) and the rows of the other ranks are not there to
        # gather, so those two status bits are expected; any other is an error
        expected = {"retrieve_merge": 0x10, "gather_rows": 0x1}
        bad = {k: v & ~expected.get(k[1], 0) for k, v in runtime.workspace_status(clear=True).items()}
        if any(bad.values()):
            raise RuntimeError(f"device status in the emulated rank: {bad}")
    else:
        runtime.raise_on_device_status()
    del step
    t.clear()
    torch.cuda.empty_cache()
    if world == 1 and not emulate and not args.no_small and w.name != "small":
        sm = small_dp_line(args, WORKLOADS["small"], dev, None, 0, 1, flush, peaks, peak_src)
        sm["config"] = run_config("small", 1, False)
        line["small_fwd_bwd"] = sm
    if rank == 0 and world == 1 and not emulate and not args.no_cpu_baseline and w.name in HOST_WORKLOADS:
        cb = cpu_baseline(w.name, args.seed, args.cpu_budget_s)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "threads", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
