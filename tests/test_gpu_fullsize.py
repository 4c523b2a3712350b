"""Parity at the benchmarked sizes, against the float64 oracle.

* small: the whole single-GPU small workload (bf16, batch 8, seq 512, d 1024,
  pool 262144 x 17408 rows, 512 lists, nprobe 8, top-k 32): the key cache of
  a row sample, the sequence means, retrieval in gate (lambda 5) and warmup
  mode with soft_full, the assembly forward and all six gradients of its VJP;
* medium: retrieval at the medium workload's shape (1M key rows, 1024
  lists, nprobe 16, top-k 64, batch 16, gate, soft_full);
* large-shaped: Zipf(1.1) lists at the large workload's list count and
  retrieval shape (4096 lists, nprobe 32, top-k 64, batch 32: the
  tensor-core scan), over 1M key rows.

Indices must equal the oracle's (tie_break="index"; each seed is checked for
a gap above 1e-6 at the list and top-k boundaries), alphas and soft_full
within rtol 1e-5, bf16 assembly outputs and gradients within rtol 2e-2, the
key cache within rtol 1e-4 (the reference test's key-cache tolerance,
tests/test_model.py:88-93).  The pool is generated on the device (9.1 GB); the
oracle reads the rows, keys and queries the kernels read.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL, BF16_TOL = 1e-5, 2e-2
f64 = np.float64


def _gaps(internals, m, k):
    c = np.sort(internals["c_score"], axis=1)[:, ::-1]
    assert (c[:, m - 1] - c[:, m] > 1e-6).all(), "seed has a near-tie among the lists"
    for b, s in enumerate(internals["s_i"]):
        s = np.sort(s)[::-1]
        assert s[k - 1] - s[k] > 1e-6, f"seed has a near-tie at the top-k boundary (query {b})"


def _host_params(rng, S, dk, d, B, T):
    f32 = np.float32
    from matrix_b200.synthetic import bf16_round
    return dict(
        W_Q=rng.standard_normal((S, dk, d), dtype=f32) * f32(d ** -0.5),
        aspect_weights=rng.standard_normal(S, dtype=f32) * f32(0.5),
        tau=f32(0.05),
        W_base=rng.standard_normal((d, d), dtype=f32) * f32(0.01),
        b_base=rng.standard_normal(d, dtype=f32) * f32(0.01),
        gamma=f32(0.1),
        h_A=bf16_round(rng.standard_normal((B, T, d), dtype=f32)),
        g_hmid=bf16_round(rng.standard_normal((B, T, d), dtype=f32) * f32(0.1)),
        g_W=rng.standard_normal((B, d, d), dtype=f32) * f32(1e-3),
    )


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def retrieval_inputs(N, C, B, seed, d, zipf=None, z_from_h=None):
    """Host inputs of a retrieval at scale: keys ~ N(0, 1/d) (the distribution
    of the key cache of pool rows ~ N(0, 1/sqrt d)), CSR lists, centroids =
    the keys of a random row per list, rich W_Q / aspect weights / tau, and
    z (random, or the mean of the given h_A)."""
    from matrix_b200.synthetic import zipf_list_offsets
    S, dk = 4, 64
    rng = np.random.default_rng(seed)
    f32 = np.float32
    keys = rng.standard_normal((S, N, dk), dtype=f32) * f32(d ** -0.5)
    off = zipf_list_offsets(N, C, zipf, rng) if zipf else np.arange(C + 1, dtype=np.int64) * (N // C)
    rows_c = off[:-1] + (rng.random(C) * np.diff(off)).astype(np.int64)
    x = dict(keys=keys, list_offsets=off, centroids=np.ascontiguousarray(keys[:, rows_c]),
             W_Q=rng.standard_normal((S, dk, d), dtype=f32) * f32(d ** -0.5),
             aspect_weights=rng.standard_normal(S, dtype=f32) * f32(0.5), tau=f32(0.05))
    x["z"] = (z_from_h.mean(axis=1, dtype=np.float64).astype(f32) if z_from_h is not None
              else rng.standard_normal((B, d), dtype=f32) * f32(0.125))
    return x


def oracle_retrieve(x, z, k, m, lam, is_warmup):
    return O.retrieve(z.astype(f64), x["W_Q"].astype(f64), x["aspect_weights"].astype(f64), f64(x["tau"]),
                      x["centroids"].astype(f64), x["keys"].astype(f64), k=k, m=m, T=1.0, lambda_val=lam,
                      is_warmup=is_warmup, list_offsets=x["list_offsets"], tie_break="index",
                      return_internals=True)


def gpu_retrieve(x, z, k, m, lam, is_warmup):
    from matrix_b200.retrieval import retrieve
    off = x["list_offsets"]
    return retrieve(z, _d(x["W_Q"]), _d(x["aspect_weights"]), torch.tensor([x["tau"]], device="cuda"),
                    _d(x["centroids"]), _d(x["keys"]), lam, is_warmup, k=k, m=m, T=1.0, list_offsets=_d(off),
                    max_list=int(np.diff(off).max()), want_soft_full=True)


SMALL_SEED = 5


def small_host(seed=SMALL_SEED):
    B, T, d, N, C = 8, 512, 1024, 262144, 512
    p = _host_params(np.random.default_rng(seed + 100), 4, 64, d, B, T)
    return p, retrieval_inputs(N, C, B, seed, d, z_from_h=p["h_A"])


def test_small_workload_end_to_end_matches_oracle():
    from matrix_b200 import _lib, runtime
    from matrix_b200.assembly import assemble_backward, assemble_forward, compute_key_cache
    B, T, d, N, C, m, k, r, S, dk = 8, 512, 1024, 262144, 512, 8, 32, 8, 4, 64
    D = d * (2 * r + 1)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    pool = torch.empty((N, D), dtype=torch.bfloat16, device=dev)
    for i in range(0, N, 16384):
        pool[i:i + 16384].normal_(0.0, d ** -0.5, generator=g)
    # the key cache of the 9.1 GB pool, checked on a row sample
    key_proj = (torch.randn((S, D, dk), generator=g, device=dev) * D ** -0.5).to(torch.bfloat16)
    keys_dev = compute_key_cache(pool, key_proj)
    rows = np.sort(np.random.default_rng(1).choice(N, 384, replace=False))
    ridx = torch.from_numpy(rows).to(dev)
    ref_keys = O.compute_key_cache(pool[ridx].double().cpu().numpy(), key_proj.double().cpu().numpy())
    assert_close(keys_dev[:, ridx].cpu().numpy(), ref_keys, 1e-4, name="key cache")
    del keys_dev, key_proj

    p, x = small_host()
    h_A = _d(p["h_A"]).to(torch.bfloat16)
    z = torch.empty((B, d), dtype=torch.float32, device=dev)
    lib = _lib.load()
    _lib.check(lib.dwa_sequence_mean(runtime.stream_of(dev), B, T, d, 1, runtime.ptr(h_A), runtime.ptr(z)),
               "dwa_sequence_mean")
    z_h = z.cpu().numpy()
    assert_close(z_h, p["h_A"].astype(f64).mean(axis=1), 1e-6, name="z")
    for is_warmup, lam in ((False, 5.0), (True, 1.0)):
        a, i, sf = gpu_retrieve(x, z, k, m, lam, is_warmup)
        ra, ri, rsf, internals = oracle_retrieve(x, z_h, k, m, lam, is_warmup)
        _gaps(internals, m, k)
        tag = "warmup" if is_warmup else "gate"
        np.testing.assert_array_equal(i.cpu().numpy(), ri, err_msg=tag)
        assert_close(a.cpu().numpy(), ra, TOL, name=f"{tag} alphas")
        assert_close(sf.cpu().numpy(), rsf, TOL, name=f"{tag} soft_full")
        if not is_warmup:
            alphas, indices = a, i
    del internals, x

    W_base, b_base, gamma = _d(p["W_base"]), _d(p["b_base"]), torch.tensor([p["gamma"]], device=dev)
    h_mid, W, W_act = assemble_forward(pool, alphas, h_A, W_base, b_base, gamma, d, r, d, row_index=indices)
    grads = assemble_backward(pool, alphas, h_A, W_act, gamma, _d(p["g_hmid"]).to(torch.bfloat16), _d(p["g_W"]),
                              d, r, d, row_index=indices)
    torch.cuda.synchronize()
    runtime.raise_on_device_status()
    gathered = pool[indices.long()].double().cpu().numpy()
    al = alphas.double().cpu().numpy()
    hA = p["h_A"].astype(f64)
    ref_h, ref_W = O.assemble(gathered, al, hA, p["W_base"].astype(f64), p["b_base"].astype(f64), f64(p["gamma"]),
                              d, r, d)
    assert_close(h_mid.float().cpu().numpy(), ref_h, BF16_TOL, name="h_mid")
    assert_close(W.cpu().numpy(), ref_W, BF16_TOL, name="W")
    ref_g = O.assemble_bwd(gathered, al, hA, ref_W, f64(p["gamma"]), p["g_hmid"].astype(f64),
                           p["g_W"].astype(f64), d, r, d, batch_chunk=2)
    for n, got, ref in zip(("g_rows", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), grads, ref_g):
        assert_close(got.float().cpu().numpy().reshape(np.shape(ref)), ref, BF16_TOL, name=n)


MEDIUM = dict(N=1 << 20, C=1024, m=16, k=64, B=16, seed=3, zipf=None)
LARGE_SHAPED = dict(N=1 << 20, C=4096, m=32, k=64, B=32, seed=4, zipf=1.1)


def _retrieval_at_scale(N, C, m, k, B, seed, zipf=None, lam=5.0):
    x = retrieval_inputs(N, C, B, seed, 2048, zipf=zipf)
    a, i, sf = gpu_retrieve(x, _d(x["z"]), k, m, lam, False)
    ra, ri, rsf, internals = oracle_retrieve(x, x["z"], k, m, lam, False)
    _gaps(internals, m, k)
    np.testing.assert_array_equal(i.cpu().numpy(), ri)
    assert_close(a.cpu().numpy(), ra, TOL, name="alphas")
    assert_close(sf.cpu().numpy(), rsf, TOL, name="soft_full")


def test_medium_retrieval_matches_oracle():
    """1M key rows, 1024 lists, nprobe 16, top-k 64, batch 16 (the 16-query scan)."""
    _retrieval_at_scale(**MEDIUM)


def test_large_shaped_zipf_retrieval_matches_oracle():
    """4096 Zipf(1.1) lists, nprobe 32, top-k 64, batch 32 (the tensor-core
    scan) over 1M key rows."""
    _retrieval_at_scale(**LARGE_SHAPED)
