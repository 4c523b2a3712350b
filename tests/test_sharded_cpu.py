"""Row-sharded retrieval, host side (no GPU).

* ``shard_rows``: contiguous ranges of whole lists covering the pool, balanced.
* The sharded protocol restated in the oracle (one rank's summary, all-gather,
  merge) equals the single-device oracle for 1-4 ranks, with an empty rank and
  with a split through the middle of a list.
* Two real ranks over gloo (world size 2, 127.0.0.1): each computes its
  summary with the oracle, ``matrix_b200.sharded.gather_summaries`` exchanges
  them, and the merge equals the single-device result on both ranks.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from matrix_b200.config import DWAConfig
from matrix_b200.sharded import shard_rows, summary_width
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O

MODES = [(True, 1.0), (False, 5.0), (False, -2.0)]


def _case(B=6, seed=31):
    cfg = DWAConfig(D=17 * 64, N=41 * 487, use_ivf=True, C=41, m=5, d_A=64, d_B=64, r=8, k_max=24,
                    S=4, d_k=64, T=1.0, gamma_init=0.1, bf16_pool=False)
    return cfg, make_inputs(cfg, B, 8, seed, variant="rich", zipf=1.1)


def _oracle_sharded(cfg, x, shards, is_warmup, lam):
    f = np.float64
    sums, slices = [], []
    for lo, hi in shards:
        sm, sl = O.retrieve_local(x.z.astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f), f(x.tau),
                                  x.centroids.astype(f), x.keys.astype(f)[:, lo:hi], row_lo=lo,
                                  k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam, is_warmup=is_warmup,
                                  list_offsets=x.list_offsets, n_global=cfg.N)
        sums.append(sm)
        slices.append(sl)
    return np.stack(sums), slices


def _oracle_full(cfg, x, is_warmup, lam):
    f = np.float64
    return O.retrieve(x.z.astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f), f(x.tau),
                      x.centroids.astype(f), x.keys.astype(f), k=cfg.k_max, m=cfg.m, T=cfg.T,
                      lambda_val=lam, is_warmup=is_warmup, list_offsets=x.list_offsets,
                      tie_break="index")


def test_shard_rows_are_whole_lists_covering_the_pool():
    _, x = _case()
    off = x.list_offsets
    for world in (1, 2, 3, 4, 7, 64):
        sh = shard_rows(off, world)
        assert len(sh) == world and sh[0][0] == 0 and sh[-1][1] == off[-1]
        for (lo, hi), (lo2, _) in zip(sh, sh[1:]):
            assert hi == lo2 and lo <= hi
        for lo, hi in sh:
            assert lo in set(off.tolist()) and hi in set(off.tolist())
    # balance: with equal lists the ranges differ by at most one list
    eq = np.arange(0, 1025, 8)
    sizes = [hi - lo for lo, hi in shard_rows(eq, 4)]
    assert max(sizes) - min(sizes) <= 8


@pytest.mark.parametrize("is_warmup,lam", MODES)
@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_oracle_protocol_equals_single_device(world, is_warmup, lam):
    cfg, x = _case()
    shards = shard_rows(x.list_offsets, world)
    sums, slices = _oracle_sharded(cfg, x, shards, is_warmup, lam)
    assert sums.shape == (world, x.z.shape[0], summary_width(cfg.k_max))
    a, i, st = O.merge_summaries(sums, k=cfg.k_max, T=cfg.T, lambda_val=lam, tau=float(x.tau),
                                 is_warmup=is_warmup)
    ra, ri, rsf = _oracle_full(cfg, x, is_warmup, lam)
    np.testing.assert_array_equal(i, ri)
    np.testing.assert_allclose(a, ra, rtol=1e-12, atol=1e-15)
    sf = np.concatenate([np.exp(sl / cfg.T - st[:, :1]) / st[:, 1:] for sl in slices], axis=1)
    np.testing.assert_allclose(sf, rsf, rtol=1e-12, atol=1e-18)


@pytest.mark.parametrize("is_warmup,lam", MODES)
def test_oracle_protocol_with_empty_rank_and_split_list(is_warmup, lam):
    cfg, x = _case()
    off = x.list_offsets
    mid = int((off[10] + off[11]) // 2)          # through the middle of list 10
    shards = [(0, 0), (0, mid), (mid, int(off[-1]))]
    sums, _ = _oracle_sharded(cfg, x, shards, is_warmup, lam)
    assert (sums[0, :, cfg.k_max:2 * cfg.k_max] == -1).all()    # the empty rank has no candidates
    a, i, _ = O.merge_summaries(sums, k=cfg.k_max, T=cfg.T, lambda_val=lam, tau=float(x.tau),
                                is_warmup=is_warmup)
    ra, ri, _ = _oracle_full(cfg, x, is_warmup, lam)
    np.testing.assert_array_equal(i, ri)
    np.testing.assert_allclose(a, ra, rtol=1e-12, atol=1e-15)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    from matrix_b200.sharded import gather_summaries
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, x = _case()
        shards = shard_rows(x.list_offsets, world)
        lo, hi = shards[rank]
        res = {}
        for is_warmup, lam in MODES:
            f = np.float64
            sm, _ = O.retrieve_local(x.z.astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f), f(x.tau),
                                     x.centroids.astype(f), x.keys.astype(f)[:, lo:hi], row_lo=lo,
                                     k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam,
                                     is_warmup=is_warmup, list_offsets=x.list_offsets, n_global=cfg.N)
            g = gather_summaries(torch.from_numpy(sm), None).numpy()
            a, i, _ = O.merge_summaries(g, k=cfg.k_max, T=cfg.T, lambda_val=lam, tau=float(x.tau),
                                        is_warmup=is_warmup)
            res[f"a_{is_warmup}_{lam}"] = a
            res[f"i_{is_warmup}_{lam}"] = i
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_and_merge(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_gloo_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    cfg, x = _case()
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npz")
        for is_warmup, lam in MODES:
            ra, ri, _ = _oracle_full(cfg, x, is_warmup, lam)
            np.testing.assert_array_equal(got[f"i_{is_warmup}_{lam}"], ri)
            np.testing.assert_allclose(got[f"a_{is_warmup}_{lam}"], ra, rtol=1e-12, atol=1e-15)
