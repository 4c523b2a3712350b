#!/usr/bin/env python
"""Benchmark of the DWA hot path on B200: retrieve + assemble + apply, with the
custom-VJP backward, on the single-GPU "small" workload
(bf16, batch 8, seq 512, d 1024, pool 262144 x 17408, 512 lists, nprobe 8,
top-k 32, gate selection with soft_full, forward + backward).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

One JSON line on rank 0.  ``value`` is assembled tokens/s of the whole job
(all ranks), timed on the device with CUDA events around each step, L2
flushed (512 MB write, then a 256 MB read) between steps, max over ranks.  One step is replayed
from a CUDA graph of: z = mean_t h_A -> dwa_retrieve -> dwa_assemble_fwd ->
dwa_assemble_bwd (+ an NCCL all-reduce of the replicated-parameter gradients
when N > 1, the shard_map transpose of the reference's batch-sharded path).
With N GPUs every rank runs its own batch against its own pool replica
(data parallel, weak scaling).

``e2e`` repeats the step through the public Python API with the step's
inputs copied from pinned host memory and its results copied back inside the
timed region.  ``--impl reference`` times the CPU restatement of the
reference's algorithm (the NumPy oracle; JAX is not installable here) on the
host cores.
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


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="small")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-budget-s", type=float, default=20.0,
                    help="CPU seconds for the cpu_baseline sample (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sharded", action="store_true",
                    help="row-shard the pool over the ranks (the medium / large configs): the "
                         "workload's batch is the global batch, each rank holds 1/N of the rows")
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="with --sharded on one GPU: run rank 0 of this many ranks (its row share, "
                         "retrieval for the whole batch over it, assembly of its sequences), no collectives")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip timing the retrieval VJP and the auxiliary losses")
    ap.add_argument("--no-key-cache", action="store_true",
                    help="skip timing compute_key_cache (once per window, not part of the step)")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# --------------------------------------------------------------- workload ---
def build_device_workload(w, device, seed):
    """Seeded synthetic inputs generated on the device (the pool is 9 GB)."""
    import torch
    cfg = w.cfg
    g = torch.Generator(device=device).manual_seed(seed)
    d, D, N, S, dk, C = cfg.d_A, cfg.D, cfg.N, cfg.S, cfg.d_k, cfg.C
    bf = torch.bfloat16
    pool = torch.empty((N, D), dtype=bf, device=device)
    step = 16384
    for i in range(0, N, step):
        pool[i:i + step].normal_(0.0, d ** -0.5, generator=g)
    key_proj = (torch.randn((S, D, dk), generator=g, device=device) * D ** -0.5).to(bf)
    from matrix_b200.assembly import compute_key_cache
    keys = compute_key_cache(pool, key_proj)        # once per window in training (outside the step)
    off = torch.arange(C + 1, dtype=torch.int64, device=device) * (N // C)
    rows = off[:-1] + torch.randint(0, N // C, (C,), generator=g, device=device)
    t = dict(
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
    return t


class Step:
    """One hot-path step on device-resident inputs through the C ABI."""

    def __init__(self, w, t, group):
        import torch
        from matrix_b200 import _lib
        self.w, self.t, self.group = w, t, group
        self.lib = _lib.load()
        self.z = torch.empty((w.batch, w.cfg.d_A), dtype=torch.float32, device=t["h_A"].device)

    def __call__(self, h_A=None, g_hmid=None, g_W=None):
        import torch
        from matrix_b200 import runtime
        from matrix_b200.assembly import assemble_backward, assemble_forward
        from matrix_b200.retrieval import retrieve
        w, t, cfg = self.w, self.t, self.w.cfg
        h_A = t["h_A"] if h_A is None else h_A
        g_hmid = t["g_hmid"] if g_hmid is None else g_hmid
        g_W = t["g_W"] if g_W is None else g_W
        dev = h_A.device
        rc = self.lib.dwa_sequence_mean(runtime.stream_of(dev), w.batch, w.seq, cfg.d_A, 1,
                                        runtime.ptr(h_A), runtime.ptr(self.z))
        from matrix_b200 import _lib
        _lib.check(rc, "dwa_sequence_mean")
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
                dist.all_reduce(flat, group=self.group)
                out["g_params"] = flat
        return out


# ------------------------------------------------- row-sharded workload ---
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
        pool=pool, keys=keys, row_lo=lo, row_hi=hi, list_offsets=torch.from_numpy(off_np).to(device),
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
    from the ranks that hold them (peer loads), their assembly and, with the
    backward, the rows' gradients returned to their owners and the parameter
    gradients all-reduced."""

    def __init__(self, w, t, group, rank, world, emulate=0):
        import torch
        from matrix_b200 import _lib
        from matrix_b200.peer import PeerPool
        self.w, self.t, self.group, self.rank, self.world = w, t, group, rank, world
        self.emulate = emulate
        self.lib = _lib.load()
        dev = t["h_A"].device
        Bp = w.batch // (emulate or world)
        if emulate:
            rank = t["rank"]
            self.z_rest = torch.empty((w.batch - Bp, w.cfg.d_A), dtype=torch.float32, device=dev)
        self.b0, self.b1 = rank * Bp, (rank + 1) * Bp
        self.z_local = torch.empty((Bp, w.cfg.d_A), dtype=torch.float32, device=dev)
        self.z = torch.empty((w.batch, w.cfg.d_A), dtype=torch.float32, device=dev)
        bounds = None
        if emulate:
            self.peers = PeerPool.from_shards([t["pool"]], [t["row_lo"], t["row_hi"]])
        elif world > 1:
            import torch.distributed as dist
            lohi = [None] * world
            dist.all_gather_object(lohi, (t["row_lo"], t["row_hi"]), group=group)
            bounds = [lohi[0][0]] + [h for _, h in lohi]
            self.peers = PeerPool(t["pool"], bounds, group)
        else:
            self.peers = PeerPool.from_shards([t["pool"]], [0, t["row_hi"]])

    def __call__(self):
        import torch
        from matrix_b200 import _lib, runtime
        from matrix_b200.assembly import assemble_backward, assemble_forward
        from matrix_b200.pool_grad import scatter_pool_grad_gathered
        from matrix_b200.sharded import RowShard, sharded_retrieve
        w, t, cfg = self.w, self.t, self.w.cfg
        dev = t["h_A"].device
        rc = self.lib.dwa_sequence_mean(runtime.stream_of(dev), self.z_local.shape[0], w.seq, cfg.d_A, 1,
                                        runtime.ptr(t["h_A"]), runtime.ptr(self.z_local))
        _lib.check(rc, "dwa_sequence_mean")
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.z, self.z_local, group=self.group)
            z = self.z
        elif self.emulate:
            # the other ranks' query means, in place of the all-gather
            Bq = w.batch - self.z_local.shape[0]
            rc = self.lib.dwa_sequence_mean(runtime.stream_of(dev), Bq, w.seq, cfg.d_A, 1,
                                            runtime.ptr(t["h_A_rest"]), runtime.ptr(self.z_rest))
            _lib.check(rc, "dwa_sequence_mean")
            self.z[: self.b0].copy_(self.z_rest[: self.b0])
            self.z[self.b0: self.b1].copy_(self.z_local)
            self.z[self.b1:].copy_(self.z_rest[self.b0:])
            z = self.z
        else:
            z = self.z_local
        alphas, indices, soft = sharded_retrieve(
            z, t["W_Q"], t["aspect_weights"], t["tau"], t["centroids"], t["keys"], t["list_offsets"], t["lam"],
            w.is_warmup, RowShard(t["row_lo"], t["row_hi"], cfg.N, self.group), k=cfg.k_max, m=cfg.m, T=cfg.T,
            max_list=t["max_list"], want_soft_full=w.soft_full)
        idx_mine = indices[self.b0:self.b1]
        rows = self.peers.gather(idx_mine)
        h_mid, W, W_act = assemble_forward(rows, alphas[self.b0:self.b1], t["h_A"], t["W_base"], t["b_base"],
                                           t["gamma"], cfg.d_B, cfg.r, cfg.d_A)
        out = dict(alphas=alphas, indices=indices, soft_full=soft, h_mid=h_mid, W=W)
        if w.backward:
            g = assemble_backward(rows, alphas[self.b0:self.b1], t["h_A"], W_act, t["gamma"], t["g_hmid"],
                                  t["g_W"], cfg.d_B, cfg.r, cfg.d_A)
            out.update(zip(("g_rows", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), g))
            scatter_pool_grad_gathered(g[0], idx_mine, t["g_pool"], row_lo=t["row_lo"], n_global=cfg.N,
                                       group=self.group)
            if self.world > 1:
                import torch.distributed as dist
                flat = torch.cat([out["g_W_base"].reshape(-1), out["g_b_base"], out["g_gamma"]])
                dist.all_reduce(flat, group=self.group)
                out["g_params"] = flat
        return out


# ------------------------------------------------------------ decode sweep ---
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

        def step():
            rc = lib.dwa_sequence_mean(runtime.stream_of(dev), B, 1, d, 1, runtime.ptr(h_A), runtime.ptr(z))
            _lib.check(rc, "dwa_sequence_mean")
            al, idx, _ = retrieve(z, W_Q, aw, tau, cent, keys, lam, False, k=k, m=c.m, T=c.T,
                                  want_soft_full=False)
            return assemble_apply(pool, al, h_A, W_base, b_base, gamma, d, r, d, row_index=idx)

        step()
        torch.cuda.synchronize()
        c0 = _lib.launch_counters()[0]
        step()
        torch.cuda.synchronize()
        launches = _lib.launch_counters()[0] - c0
        kms, _ = profile_kernels(step, flush)
        s_ = torch.cuda.Stream()
        s_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_):
            step()
        torch.cuda.current_stream().wait_stream(s_)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(max(args.warmup, 3)):
            flush()
            graph.replay()
        reps = 20
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        torch.cuda.synchronize()
        for a, b in ev:
            flush()
            a.record()
            graph.replay()
            b.record()
        torch.cuda.synchronize()
        ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
        del graph
        runtime.raise_on_device_status()
        row_bytes = B * k * D * 2
        pt = {"batch": B, "top_k": k, "ms_per_token_step": ms, "tokens_per_s": B / (ms / 1e3),
              "kernels_ms": kms, "gpu_launches_per_step": int(launches),
              "gathered_row_bytes": row_bytes}
        # the two row kernels each read their part of every winning row
        for name, part in (("factored_hv", r * d), ("factored_out", d * r + d)):
            if kms.get(name):
                gbs = B * k * part * 2 / (kms[name] / 1e3) / 1e9
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
                       "l2": "flushed between steps (512 MB write, then 256 MB read)",
                       "step": "CUDA graph: seq_mean + dwa_retrieve + dwa_assemble_apply",
                       "headline": "batch 256, top-k 128"},
            "peak_hbm_gbs": float(peaks["hbm_gbs"]), "peak_source": peak_src, "sweep": points}


# ------------------------------------------------------ roofline numbers ---
def profiled_traffic(kernel, w):
    """DRAM bytes (read + write) per launch of `kernel` at workload `w`, from
    the `traffic:` lines of the ncu summaries under profiles/.  A summary
    captured on a smaller case is scaled by the queries x pool rows it
    processed (the key stream and the s_full writes both grow with them)."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
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
                scale = (w.cfg.N * w.batch) / (float(kv["rows"]) * float(kv["queries"]))
                return int((int(kv["dram_read_bytes"]) + int(kv["dram_write_bytes"])) * scale)
    return None


def kernel_work(w, name, n_rows=None, seqs=None):
    """Algorithmic bytes (HBM-bound kernels) or flops (tensor kernels) of one
    launch of `name` on workload w; returns (bound, amount).  A rank of a
    row-sharded pool scores ``n_rows`` rows for all ``w.batch`` queries and
    assembles ``seqs`` sequences."""
    c = w.cfg
    B, T, d, k, r, S, dk, N = w.batch, w.seq, c.d_A, c.k_max, c.r, c.S, c.d_k, c.N
    N = N if n_rows is None else n_rows
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
    }
    return table.get(name, ("hbm", None))


KERNELS = ["seq_mean", "query", "query_norm", "coarse", "topm", "full_scores", "fine", "select",
           "softmax_stats",
           "softmax_apply", "prep_factors", "prep_bias", "gemm_W", "gemm_apply", "gemm_G",
           "gemm_gh", "gemm_P", "gemm_Q", "colsum", "finalize", "bias_grad", "merge", "gather_rows",
           "factored_hv", "base_rows", "cast_w_base", "gemm_base", "factored_out", "factored_combine", "probe_lists"]


def profile_kernels(step, flush, n=5):
    """Average duration (ms) of every library kernel of one step, and its start
    relative to the step's first kernel (the sequence mean), from replays of a
    CUDA graph of the step in which the library records an event pair around
    each kernel (no host launch gaps inside the measurement).  A kernel the
    step does not launch keeps its setup record, which precedes the replay."""
    import torch
    from matrix_b200 import _lib
    lib = _lib.load()
    ev = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for k in KERNELS}
    for a, b in ev.values():     # torch creates the CUDA event on its first record
        a.record(); b.record()
    torch.cuda.synchronize()
    for k, (a, b) in ev.items():
        lib.dwa_profile_kernel(k.encode(), C_ptr(a), C_ptr(b))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    lib.dwa_profile_clear()
    first = ev[KERNELS[0]][0]
    acc = {k: [] for k in KERNELS}
    start = {k: [] for k in KERNELS}
    for _ in range(n):
        flush()
        g.replay()
        torch.cuda.synchronize()
        for k, (a, b) in ev.items():
            t0 = first.elapsed_time(a)
            if t0 >= 0.0:
                acc[k].append(a.elapsed_time(b))
                start[k].append(t0)
    del g
    dur = {k: float(np.mean(v)) for k, v in acc.items() if v}
    return dur, {k: float(np.mean(start[k])) for k in dur}


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
    """The training-time parts next to the step, on the workload's inputs, timed
    with CUDA events after a flush (best of ``reps``):

    * ``retrieve_bwd``: the retrieval VJP for the alphas' cotangent alone (the
      key pass visits only the probed lists' tiles), with the soft_full
      cotangent as well (the key pass reads every key row), and with the
      key-cache gradient; the key pass of the full case against the HBM
      roofline (keys + G read once: 4 (S N d_k + B N) bytes);
    * ``aux_losses``: the four losses and their gradients.
    The cotangents are seeded synthetic values of the right shapes."""
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
    keys_ms, _ = timed(lambda: bwd(g_sf, True))
    S, N, dk = t["keys"].shape
    B = z.shape[0]
    kp_bytes = 4.0 * (S * N * dk + B * N)
    out = {"retrieve_bwd": {
        "alphas_only_ms": probed_ms, "alphas_and_soft_full_ms": full_ms, "with_key_grad_ms": keys_ms,
        "key_pass": {"kernel": "key_grad", "ms": kp_ms, "algorithmic_bytes": kp_bytes,
                     "hbm_gbs": kp_bytes / (kp_ms * 1e-3) / 1e9 if kp_ms else None,
                     "frac": (kp_bytes / (kp_ms * 1e-3) / 1e9) / float(peaks["hbm_gbs"]) if kp_ms else None},
        "shape": f"B {B}, keys [{S}, {N}, {dk}] f32, {cfg.m} probes of {cfg.N // cfg.C} rows, top-k {cfg.k_max}"}}
    W = torch.randn((B, cfg.d_B, cfg.d_A), generator=g, device=z.device) * 0.01
    aux_ms, _ = timed(lambda: aux_losses_and_grads(alphas, indices, t["keys"], W, t["W_base"], soft_full))
    out["aux_losses"] = {"ms": aux_ms, "shape": f"B {B}, k {cfg.k_max}, N {N}, W [{B}, {cfg.d_B}, {cfg.d_A}] f32"}
    return out


def C_ptr(event):
    import ctypes
    return ctypes.c_void_p(event.cuda_event)


# ---------------------------------------------------------------- clocks ---
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
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
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------- CPU baseline ---
def cpu_baseline(w, t, budget_s):
    """The NumPy oracle (the reference's algorithm, float32) on one sequence of
    the same workload per sample, with the same key cache and pool rows."""
    from oracle import dwa_oracle as O
    import torch
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        threads = 1
    cfg = w.cfg
    keys = t["keys"].cpu().numpy()
    cents = t["centroids"].cpu().numpy()
    W_Q = t["W_Q"].cpu().numpy()
    aw = t["aspect_weights"].cpu().numpy()
    W_base = t["W_base"].cpu().numpy()
    b_base = t["b_base"].cpu().numpy()
    gamma = np.float32(t["gamma"].item())
    h_all = t["h_A"].float().cpu().numpy()
    g_all = t["g_hmid"].float().cpu().numpy()
    gW_all = t["g_W"].cpu().numpy()
    pool = t["pool"]

    def one(b):
        h = h_all[b:b + 1]
        z = h.mean(axis=1, dtype=np.float32)
        a, idx, sf = O.retrieve(z, W_Q, aw, np.float32(0.0), cents, keys, k=cfg.k_max, m=cfg.m,
                                T=cfg.T, lambda_val=w.lambda_val, is_warmup=w.is_warmup,
                                want_soft_full=w.soft_full)
        gathered = pool[torch.from_numpy(idx).to(pool.device)].float().cpu().numpy()
        h_mid, W = O.assemble(gathered, a, h, W_base, b_base, gamma, cfg.d_B, cfg.r, cfg.d_A)
        if w.backward:
            O.assemble_bwd(gathered, a, h, W, gamma, g_all[b:b + 1], gW_all[b:b + 1],
                           cfg.d_B, cfg.r, cfg.d_A)

    one(0)  # warm-up
    times, b = [], 0
    t0 = time.perf_counter()
    while not times or (time.perf_counter() - t0 < budget_s and len(times) < w.batch):
        s = time.perf_counter()
        one(b % w.batch)
        times.append(time.perf_counter() - s)
        b += 1
    sec_per_seq = float(np.mean(times))
    return {"value": w.seq / sec_per_seq, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} of {w.batch} sequences ({w.seq} tokens each): NumPy float32 "
                      f"oracle of retrieval.py:48-159 + model.py:193-195 + assemble_jax + "
                      f"_pallas_assemble_bwd, same key cache and pool rows as the GPU run",
            "sec_per_sequence": sec_per_seq}


def reference_arm(args, w, rank):
    """--impl reference: the CPU port timed per step on one sequence per step."""
    if rank != 0:
        return
    import torch
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    if dev is None:
        print(json.dumps({"impl": "reference", "unavailable": "needs the device workload builder"}))
        return
    t = build_device_workload(w, dev, args.seed)
    budget = 150.0
    cb = cpu_baseline(w, t, budget_s=min(budget, 30.0))
    sec = cb["sec_per_sequence"]
    steps = int(min(args.steps, max(1, budget // max(sec, 1e-9))))
    value = cb["value"]
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "steps_requested": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w.name, "note": w.note},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- main ---
def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    from matrix_b200.config import WORKLOADS
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        return reference_arm(args, w, rank)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD

    flush_buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        # write 512 MB (> 126 MB L2), then read back 256 MB of it: the write
        # evicts the step's data, the read makes the flush's dirty lines be
        # written back here rather than inside the next timed step
        flush_buf.zero_()
        flush_sink.copy_(flush_buf[: flush_buf.numel() // 2].sum())

    if w.name in ("decode", "decode_profile") and not args.sharded:
        # the decode pool (2M x 69632, 292 GB) needs 8 GPUs; one GPU runs one rank's share
        if world > 1:
            raise SystemExit("the decode sweep runs on one GPU (one rank's share of the pool)")
        peaks, peak_src = load_peaks()
        print(json.dumps(decode_sweep(args, w, dev, flush, peaks, peak_src)), flush=True)
        return

    if args.sharded:
        # a manual mode for the configs whose pool is row-sharded; the driver's
        # runs use the data-parallel default
        args.no_e2e = args.no_extras = args.no_key_cache = args.no_cpu_baseline = True
        if args.emulate_ranks and world > 1:
            raise SystemExit("--emulate-ranks runs on one GPU")
        t = build_sharded_workload(w, dev, rank, world, group, args.seed, emulate=args.emulate_ranks)
        step = ShardedStep(w, t, group, rank, world, emulate=args.emulate_ranks)
    else:
        t = build_device_workload(w, dev, args.seed + rank)
        step = Step(w, t, group)

    from matrix_b200 import _lib
    step()                       # first call: workspaces, kernel attributes
    torch.cuda.synchronize()
    c0 = _lib.launch_counters()[0]
    step()
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_counters()[0] - c0

    breakdown, kstarts = profile_kernels(step, flush)
    dominant = max(breakdown, key=breakdown.get)

    # capture the step in a CUDA graph, with the dominant kernel's events inside
    lib = _lib.load()
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record(); kb.record()     # the library re-records both inside every graph replay
    torch.cuda.synchronize()
    lib.dwa_profile_kernel(dominant.encode(), C_ptr(ka), C_ptr(kb))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    lib.dwa_profile_clear()

    for _ in range(max(args.warmup, 3)):
        flush()
        graph.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                           else local)
    sampler.start()
    time.sleep(0.2)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kern_ms = []
    kern_src = "graph replay (external event nodes)"
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush()
        starts[i].record()
        graph.replay()
        stops[i].record()
        stops[i].synchronize()
        if kern_src is not None:
            try:
                kern_ms.append(ka.elapsed_time(kb))
            except Exception:  # noqa: BLE001  (no timing on graph-recorded events)
                kern_src, kern_ms = None, []
    torch.cuda.synchronize()
    if group is not None:
        dist.barrier()
    clocks = sampler.stop()
    if kern_src is None:
        # time the dominant kernel's launches in eager steps, same flush discipline
        kern_src = "eager steps"
        ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ka.record(); kb.record()
        lib.dwa_profile_kernel(dominant.encode(), C_ptr(ka), C_ptr(kb))
        for i in range(min(args.steps, 50)):
            flush()
            step()
            torch.cuda.synchronize()
            kern_ms.append(ka.elapsed_time(kb))
        lib.dwa_profile_clear()
    step_ms = float(sum(a.elapsed_time(b) for a, b in zip(starts, stops)))
    tmax = torch.tensor([step_ms], device=dev, dtype=torch.float64)
    if group is not None:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    total_ms = float(tmax.item())
    ms_per_step = total_ms / args.steps
    tokens = w.batch * w.seq
    if args.emulate_ranks:      # this GPU's sequences: rank 0's share of the batch
        tokens = w.batch // args.emulate_ranks * w.seq
    # data parallel: w.batch sequences per rank; row-sharded: w.batch in all
    value = tokens * (1 if args.sharded else world) / (ms_per_step / 1e3)

    # ---- end to end through the public API with pinned host buffers ----
    e2e = None
    if not args.no_e2e:
        hA_h = t["h_A"].cpu().pin_memory()
        g_h = t["g_hmid"].cpu().pin_memory()
        gW_h = t["g_W"].cpu().pin_memory()
        hA_d, g_d, gW_d = torch.empty_like(t["h_A"]), torch.empty_like(t["g_hmid"]), torch.empty_like(t["g_W"])
        res_keys = ["h_mid", "g_hA", "g_rows", "g_alpha", "g_W_base", "g_b_base", "g_gamma",
                    "alphas", "indices"]
        out = step(hA_d.copy_(hA_h), g_d.copy_(g_h), gW_d.copy_(gW_h))
        pinned = {k: torch.empty(out[k].shape, dtype=out[k].dtype).pin_memory() for k in res_keys}
        h2d = hA_h.nbytes + g_h.nbytes + gW_h.nbytes
        d2h = sum(v.nbytes for v in pinned.values())
        n_e2e = min(args.steps, 50)
        # A training loop's input pipeline: step i+1's inputs go up on a copy
        # stream while step i computes and step i-1's results come down on
        # another; device inputs and pinned host outputs are double-buffered.
        # Every step's H2D and D2H is inside the timed region; L2 is not flushed
        # (the pool and key cache are larger than L2).
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        main = torch.cuda.current_stream()
        bufs = [(hA_d, g_d, gW_d), (torch.empty_like(hA_d), torch.empty_like(g_d), torch.empty_like(gW_d))]
        pins = [pinned, {k: torch.empty_like(v).pin_memory() for k, v in pinned.items()}]
        ev_in = [torch.cuda.Event() for _ in range(n_e2e)]
        ev_used = [torch.cuda.Event() for _ in range(n_e2e)]
        ev_out = [torch.cuda.Event() for _ in range(n_e2e)]
        t_start, t_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ring = [None, None]     # step outputs alive until their copy to the host is done
        t_start.record(main)
        s_in.wait_event(t_start)
        for i in range(n_e2e):
            bh, bg, bw = bufs[i % 2]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_used[i - 2])      # step i-2 has read this buffer
                bh.copy_(hA_h, non_blocking=True)
                bg.copy_(g_h, non_blocking=True)
                bw.copy_(gW_h, non_blocking=True)
                ev_in[i].record(s_in)
            main.wait_event(ev_in[i])
            if i >= 2:
                # step i-2's outputs reached the host: release them in stream order
                main.wait_event(ev_out[i - 2])
                ring[i % 2] = None
            out = step(bh, bg, bw)
            ev_used[i].record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[i])
                for k in res_keys:
                    pins[i % 2][k].copy_(out[k], non_blocking=True)
                ev_out[i].record(s_out)
            ring[i % 2] = out
        main.wait_event(ev_out[n_e2e - 1])
        t_stop.record(main)
        t_stop.synchronize()
        e_ms = torch.tensor([t_start.elapsed_time(t_stop) / n_e2e], device=dev, dtype=torch.float64)
        if group is not None:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": tokens * world / (float(e_ms.item()) / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": float(e_ms.item()), "steps": n_e2e,
               "mode": "copies overlapped with compute on two copy streams, double-buffered; "
                       "no L2 flush (inputs larger than L2)"}

    # ---- roofline of the dominant kernel ----
    peaks, peak_src = load_peaks()
    if args.sharded:
        bound, work = kernel_work(w, dominant, n_rows=t["row_hi"] - t["row_lo"],
                                  seqs=w.batch // (args.emulate_ranks or world))
    else:
        bound, work = kernel_work(w, dominant)
    kms = float(np.mean(kern_ms))
    roof = None
    if work is not None:
        if bound == "hbm":
            ach = work / (kms / 1e3) / 1e9
            peak = float(peaks["hbm_gbs"])
            unit = "GB/s"
        else:
            ach = work / (kms / 1e3) / 1e12
            peak = float(peaks["bf16_tflops"])
            unit = "TFLOP/s"
        traffic = None if args.sharded else profiled_traffic(dominant, w)
        roof = {"kernel": dominant, "bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                "frac": ach / peak, "traffic": traffic, "peak_source": peak_src,
                "algorithmic_per_launch": work, "launch_ms": kms, "timed_in": kern_src}

    if args.sharded:
        step_desc = ("CUDA graph: seq_mean + all-gather of z + dwa_retrieve_local + all-gather of summaries + "
                     "dwa_retrieve_merge + dwa_gather_rows (peer loads) + dwa_assemble_fwd"
                     + (" + dwa_assemble_bwd + pool-row gradient all-gather and scatter + NCCL all_reduce of "
                        "parameter grads" if w.backward else ""))
    else:
        step_desc = ("CUDA graph: seq_mean + dwa_retrieve + dwa_assemble_fwd + dwa_assemble_bwd"
                     + (" + NCCL all_reduce of parameter grads" if world > 1 else ""))
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if args.sharded else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": w.name, "note": w.note,
                       "global_batch": w.batch if args.sharded else w.batch * world,
                       "seq_len": w.seq, "parallelism": f"rows{world}" if args.sharded else f"dp{world}",
                       "mode": "warmup" if w.is_warmup else f"gate lambda={w.lambda_val}",
                       "soft_full": w.soft_full, "backward": w.backward,
                       "l2": "flushed between steps (512 MB write, then 256 MB read)",
                       "step": step_desc},
            "value_per_gpu": value / world, "roofline": roof,
            "kernels_ms": breakdown, "kernels_start_ms": kstarts, "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clocks, "e2e": e2e}
    if args.emulate_ranks:
        P = args.emulate_ranks
        line["config"]["parallelism"] = f"rows{P}, one rank emulated on one GPU"
        line["config"]["emulated"] = (
            f"rank {t['rank']} of {P} (the most rows): pool rows [{t['row_lo']}, {t['row_hi']}) of {w.cfg.N} (whole lists), retrieval of "
            f"all {w.batch} queries over them, assembly of its {w.batch // P} sequences; the all-gathers, the "
            f"merge across ranks, peer reads and the row-gradient exchange are not in it")
        line["value_per_gpu"] = value
    if world == 1 and not args.no_key_cache:
        line["key_cache"] = time_key_cache(t, flush, peaks)
    if world == 1 and not args.no_extras:
        line.update(time_training_extras(w, t, flush, peaks))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(w, t, args.cpu_budget_s)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if group is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
