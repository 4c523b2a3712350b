"""Row-sharded retrieval on the GPU through the C ABI.

Ranks are emulated on one GPU: each rank's ``dwa_retrieve_local`` runs on its
own slice of the key cache, the summaries are stacked as an all-gather would
stack them, and every rank's ``dwa_retrieve_merge`` must give the indices of
``dwa_retrieve`` on the whole pool bit-exactly (and the oracle's), alphas and
the concatenated soft_full slices within rtol 1e-5.  Cases: 2 and 3 ranks,
warmup and both gate signs, Zipf lists, an empty rank, a split through the
middle of a list, full search (IVF off).  With two or more GPUs visible, two
NCCL ranks also run ``sharded_retrieve`` for real.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5
MODES = [(True, 1.0), (False, 5.0), (False, -2.0)]


def _case(B=6, seed=31):
    cfg = DWAConfig(D=17 * 64, N=41 * 487, use_ivf=True, C=41, m=5, d_A=64, d_B=64, r=8, k_max=24,
                    S=4, d_k=64, T=1.0, gamma_init=0.1, bf16_pool=False)
    return cfg, make_inputs(cfg, B, 8, seed, variant="rich", zipf=1.1)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _emulated(cfg, x, shards, is_warmup, lam, use_ivf=True, want_sf=True):
    from matrix_b200.sharded import retrieve_local, retrieve_merge
    z, W_Q, aw = _dev(x.z), _dev(x.W_Q), _dev(x.aspect_weights)
    tau, cents, off = torch.tensor(x.tau).cuda(), _dev(x.centroids), _dev(x.list_offsets)
    keys = _dev(x.keys)
    max_list = int(np.diff(x.list_offsets).max())
    sums, softs = [], []
    for lo, hi in shards:
        local = keys[:, lo:hi].contiguous()
        sm, sf = retrieve_local(z, W_Q, aw, tau, cents, local, off, lam, is_warmup, k=cfg.k_max,
                                m=cfg.m, T=cfg.T, row_lo=lo, n_global=cfg.N, max_list=max_list,
                                use_ivf=use_ivf, want_soft_full=want_sf)
        sums.append(sm)
        softs.append(sf)
    gathered = torch.stack(sums)
    outs = []
    for p in range(len(shards)):
        a, i = retrieve_merge(gathered, lam, tau, is_warmup, k=cfg.k_max, T=cfg.T, soft_full=softs[p])
        outs.append((a, i))
    torch.cuda.synchronize()
    sf = torch.cat(softs, dim=1).cpu().numpy() if want_sf else None
    return [(a.cpu().numpy(), i.cpu().numpy()) for a, i in outs], sf


def _single(cfg, x, is_warmup, lam, use_ivf=True, want_sf=True):
    from matrix_b200.retrieval import retrieve
    a, i, sf = retrieve(_dev(x.z), _dev(x.W_Q), _dev(x.aspect_weights), torch.tensor(x.tau).cuda(),
                        _dev(x.centroids), _dev(x.keys), lam, is_warmup, k=cfg.k_max, m=cfg.m, T=cfg.T,
                        use_ivf=use_ivf, list_offsets=_dev(x.list_offsets),
                        max_list=int(np.diff(x.list_offsets).max()), want_soft_full=want_sf)
    torch.cuda.synchronize()
    return a.cpu().numpy(), i.cpu().numpy(), None if sf is None else sf.cpu().numpy()


def _check(cfg, x, shards, is_warmup, lam, use_ivf=True, want_sf=True):
    from matrix_b200.runtime import raise_on_device_status
    outs, sf = _emulated(cfg, x, shards, is_warmup, lam, use_ivf, want_sf)
    ra, ri, rsf = _single(cfg, x, is_warmup, lam, use_ivf, want_sf)
    f = np.float64
    oa, oi, _ = O.retrieve(x.z.astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f), f(x.tau),
                           x.centroids.astype(f), x.keys.astype(f), k=cfg.k_max, m=cfg.m, T=cfg.T,
                           lambda_val=lam, is_warmup=is_warmup, use_ivf=use_ivf,
                           list_offsets=x.list_offsets, tie_break="index", want_soft_full=False)
    tag = f"shards={shards} warmup={is_warmup} lam={lam} ivf={use_ivf}"
    for p, (a, i) in enumerate(outs):
        np.testing.assert_array_equal(i, ri, err_msg=f"rank {p} vs single call, {tag}")
        assert_close(a, ra, TOL, name=f"alphas rank {p} {tag}")
        if is_warmup or lam >= 0:
            np.testing.assert_array_equal(i, oi, err_msg=f"rank {p} vs oracle, {tag}")
            assert_close(a, oa, TOL, name=f"alphas rank {p} vs oracle {tag}")
    if want_sf:
        assert_close(sf, rsf, TOL, name=f"soft_full {tag}")
    raise_on_device_status()


@pytest.mark.parametrize("is_warmup,lam", MODES)
@pytest.mark.parametrize("world", [2, 3])
def test_emulated_ranks_equal_single_call(world, is_warmup, lam):
    from matrix_b200.sharded import shard_rows
    cfg, x = _case()
    _check(cfg, x, shard_rows(x.list_offsets, world), is_warmup, lam)


@pytest.mark.parametrize("is_warmup,lam", MODES)
def test_empty_rank_and_split_list(is_warmup, lam):
    cfg, x = _case()
    off = x.list_offsets
    mid = int((off[10] + off[11]) // 2)
    _check(cfg, x, [(0, 0), (0, mid), (mid, int(off[-1]))], is_warmup, lam)


def test_without_soft_full_and_full_search():
    from matrix_b200.sharded import shard_rows
    cfg, x = _case()
    shards = shard_rows(x.list_offsets, 2)
    _check(cfg, x, shards, False, 5.0, want_sf=False)
    _check(cfg, x, shards, True, 1.0, use_ivf=False)


@pytest.mark.parametrize("k", [24, 128])
def test_many_queries_without_soft_full(k):
    """The decode shape over emulated ranks: 40 queries (more than the key
    scans take: the list-inverted fine pass in each rank's window), no
    soft_full, top-k up to 128; every rank's merge equals the single call."""
    from dataclasses import replace
    from matrix_b200.runtime import raise_on_device_status
    from matrix_b200.sharded import shard_rows
    cfg, x = _case(B=40, seed=35)
    cfg = replace(cfg, k_max=k)
    shards = shard_rows(x.list_offsets, 3)
    outs, _ = _emulated(cfg, x, shards, False, 5.0, want_sf=False)
    ra, ri, _ = _single(cfg, x, False, 5.0, want_sf=False)
    for p, (a, i) in enumerate(outs):
        # every row's score is the same computation in both calls: bit-equal ranking
        np.testing.assert_array_equal(i, ri, err_msg=f"rank {p} vs single call")
        assert_close(a, ra, TOL, name=f"alphas rank {p}")
    raise_on_device_status()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    from matrix_b200.sharded import RowShard, shard_rows, sharded_retrieve
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg, x = _case()
        lo, hi = shard_rows(x.list_offsets, world)[rank]

        def d(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        res = {}
        for is_warmup, lam in MODES:
            a, i, sf = sharded_retrieve(d(x.z), d(x.W_Q), d(x.aspect_weights), torch.tensor(x.tau).to(dev),
                                        d(x.centroids), d(x.keys[:, lo:hi]), d(x.list_offsets), lam,
                                        is_warmup, RowShard(lo, hi, cfg.N, None), k=cfg.k_max, m=cfg.m,
                                        T=cfg.T)
            torch.cuda.synchronize(dev)
            res[f"a_{is_warmup}_{lam}"] = a.cpu().numpy()
            res[f"i_{is_warmup}_{lam}"] = i.cpu().numpy()
            res[f"sf_{is_warmup}_{lam}"] = sf.cpu().numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_nccl_ranks(tmp_path):
    import torch.multiprocessing as mp
    from matrix_b200.sharded import shard_rows
    world = 2
    mp.start_processes(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    cfg, x = _case()
    shards = shard_rows(x.list_offsets, world)
    for is_warmup, lam in MODES:
        ra, ri, rsf = _single(cfg, x, is_warmup, lam)
        sfs = []
        for rank in range(world):
            got = np.load(tmp_path / f"rank{rank}.npz")
            np.testing.assert_array_equal(got[f"i_{is_warmup}_{lam}"], ri)
            assert_close(got[f"a_{is_warmup}_{lam}"], ra, TOL, name="alphas")
            sfs.append(got[f"sf_{is_warmup}_{lam}"])
        assert_close(np.concatenate(sfs, axis=1), rsf, TOL, name="soft_full")
        assert sum(hi - lo for lo, hi in shards) == cfg.N


def _peer_rank(rank, world, port, out_dir):
    """One rank of a row-sharded pool: map the peer's shard by IPC, gather the
    winning rows of this rank's sequences from both shards, assemble them, and
    return the rows' gradients to their owners (all-gather + sorted scatter,
    and peer stores into the owners' receive areas + each owner's scatter)."""
    import torch.distributed as dist
    from datetime import timedelta
    from matrix_b200.assembly import assemble_backward, assemble_forward
    from matrix_b200.peer import PeerPool
    from matrix_b200.pool_grad import PoolGradExchange, scatter_pool_grad_gathered
    from test_gpu_assembly import _setup
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    pp = None
    try:
        cfg, x, idx, alphas = _setup("bf16_small_like")
        N, B = x.pool.shape[0], idx.shape[0]
        bounds = [N * r // world for r in range(world + 1)]
        lo, hi = bounds[rank], bounds[rank + 1]

        def d(a, dt=None):
            t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            return t.to(dt) if dt is not None else t

        local = d(x.pool[lo:hi], torch.bfloat16)
        pp = PeerPool(local, bounds)
        b0, b1 = B * rank // world, B * (rank + 1) // world      # this rank's sequences
        rows = pp.gather(d(idx[b0:b1]))
        h_A = d(x.h_A[b0:b1], torch.bfloat16)
        args = (d(alphas[b0:b1]), h_A, d(x.W_base), d(x.b_base), torch.tensor(x.gamma).to(dev))
        h_mid, W, W_act = assemble_forward(rows, *args, cfg.d_B, cfg.r, cfg.d_A)
        g_rows = assemble_backward(rows, args[0], h_A, W_act, args[4], d(x.g_hmid[b0:b1], torch.bfloat16),
                                   d(x.g_W[b0:b1]), cfg.d_B, cfg.r, cfg.d_A)[0]
        g_pool = torch.zeros((hi - lo, x.pool.shape[1]), dtype=torch.float32, device=dev)
        scatter_pool_grad_gathered(g_rows, d(idx[b0:b1]), g_pool, row_lo=lo, n_global=N)
        # the same gradients returned to their owners by peer stores (bf16
        # rows), twice: the second call goes through the other receive areas
        ex = PoolGradExchange(bounds, (b1 - b0) * idx.shape[1], x.pool.shape[1], dev)
        g_pool2 = torch.zeros_like(g_pool)
        ex(g_rows, d(idx[b0:b1]), g_pool2)
        once = g_pool2.clone()
        ex(g_rows, d(idx[b0:b1]), g_pool2)
        torch.cuda.synchronize(dev)
        ex.close()
        np.savez(os.path.join(out_dir, f"peer{rank}.npz"), rows=rows.float().cpu().numpy(),
                 h_mid=h_mid.float().cpu().numpy(), W=W.cpu().numpy(), g_pool=g_pool.cpu().numpy(),
                 g_pool_owner=once.cpu().numpy(), g_pool_owner2=g_pool2.cpu().numpy())
        dist.barrier()
    finally:
        if pp is not None:
            pp.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_ranks_peer_gather_and_sharded_assembly(tmp_path):
    """Rows read over NVLink from the owning rank equal the single-device
    gather; each rank's assembly of its sequences equals the single-device
    assembly; the owners' scattered row gradients equal the single-device
    pool gradient."""
    import torch.multiprocessing as mp
    from matrix_b200.assembly import assemble_backward, assemble_forward
    from matrix_b200.pool_grad import scatter_pool_grad
    from test_gpu_assembly import _setup
    world = 2
    mp.start_processes(_peer_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    cfg, x, idx, alphas = _setup("bf16_small_like")
    pool = _dev(x.pool).to(torch.bfloat16)
    idx_t = _dev(idx)
    h_A = _dev(x.h_A).to(torch.bfloat16)
    args = (_dev(alphas), h_A, _dev(x.W_base), _dev(x.b_base), torch.tensor(x.gamma).cuda())
    h_mid, W, W_act = assemble_forward(pool, *args, cfg.d_B, cfg.r, cfg.d_A, row_index=idx_t)
    g_rows = assemble_backward(pool, args[0], h_A, W_act, args[4], _dev(x.g_hmid).to(torch.bfloat16),
                               _dev(x.g_W), cfg.d_B, cfg.r, cfg.d_A, row_index=idx_t)[0]
    g_pool = torch.zeros(pool.shape, dtype=torch.float32, device="cuda")
    scatter_pool_grad(g_rows, idx_t, g_pool)
    torch.cuda.synchronize()
    B, N = idx.shape[0], x.pool.shape[0]
    got = [np.load(tmp_path / f"peer{r}.npz") for r in range(world)]
    np.testing.assert_array_equal(np.concatenate([g["rows"] for g in got]),
                                  pool[idx_t.long()].float().cpu().numpy())
    np.testing.assert_array_equal(np.concatenate([g["h_mid"] for g in got]), h_mid.float().cpu().numpy())
    np.testing.assert_array_equal(np.concatenate([g["W"] for g in got]), W.cpu().numpy())
    assert_close(np.concatenate([g["g_pool"] for g in got]), g_pool.cpu().numpy(), TOL, name="g_pool")
    # bf16 transport of the row gradients: the bf16 tolerance
    owner = np.concatenate([g["g_pool_owner"] for g in got])
    assert_close(owner, g_pool.cpu().numpy(), 2e-2, name="g_pool by owner exchange")
    np.testing.assert_array_equal(np.concatenate([g["g_pool_owner2"] for g in got]), 2 * owner)


# ---------------------------------------------------------------------------
# The retrieval VJP over the same emulated ranks
# ---------------------------------------------------------------------------

def _emulated_bwd(cfg, x, shards, is_warmup, lam, g_alphas, g_soft, use_ivf=True, want_keys=True):
    """Every rank's phase 1, the sum over the ranks (the all-reduce), every
    rank's phase 2, the sum, and phase 3; the ranks' key gradients stacked."""
    from matrix_b200.retrieval import retrieve
    from matrix_b200.sharded import (bwd_workspace, retrieve_bwd_finish, retrieve_bwd_local1,
                                     retrieve_bwd_local2)
    z, W_Q, aw = _dev(x.z), _dev(x.W_Q), _dev(x.aspect_weights)
    tau, cents, off = torch.tensor(x.tau).cuda(), _dev(x.centroids), _dev(x.list_offsets)
    keys = _dev(x.keys)
    max_list = int(np.diff(x.list_offsets).max())
    kw = dict(k=cfg.k_max, m=cfg.m, T=cfg.T, max_list=max_list, use_ivf=use_ivf)
    a, i, sf = retrieve(z, W_Q, aw, tau, cents, keys, lam, is_warmup, k=cfg.k_max, m=cfg.m, T=cfg.T,
                        use_ivf=use_ivf, list_offsets=off if use_ivf else None,
                        max_list=max_list if use_ivf else None, want_soft_full=True)
    ga, gs = _dev(g_alphas), _dev(g_soft)
    C = cfg.C if use_ivf else 1
    wss, locs = [], []
    for lo, hi in shards:
        wss.append(bwd_workspace(z, W_Q, hi - lo, k=cfg.k_max, m=cfg.m, T=cfg.T, C=C, max_list=max_list,
                                 use_ivf=use_ivf))
        locs.append(keys[:, lo:hi].contiguous())
    p1 = sum(retrieve_bwd_local1(wss[r], z, W_Q, aw, tau, cents, locs[r], off, lam, is_warmup, i,
                                 sf[:, lo:hi].contiguous(), gs[:, lo:hi].contiguous(), row_lo=lo, n_global=cfg.N,
                                 **kw)
             for r, (lo, hi) in enumerate(shards))
    parts, gks = [], []
    for r, (lo, hi) in enumerate(shards):
        p2, gk = retrieve_bwd_local2(wss[r], z, W_Q, aw, tau, cents, locs[r], off, lam, is_warmup, a, i,
                                     sf[:, lo:hi].contiguous(), ga, gs[:, lo:hi].contiguous(), p1, row_lo=lo,
                                     want_key_grad=want_keys, **kw)
        parts.append(p2)
        gks.append(gk)
    out = retrieve_bwd_finish(wss[0], z, W_Q, aw, sum(parts), k=cfg.k_max, m=cfg.m, T=cfg.T, C=C,
                              max_list=max_list, use_ivf=use_ivf)
    torch.cuda.synchronize()
    res = {k_: v.cpu().numpy() for k_, v in out.items()}
    if want_keys:
        res["g_pool_keys"] = torch.cat(gks, dim=1).cpu().numpy()
    return res, (a, i, sf)


@pytest.mark.parametrize("is_warmup,lam", [(True, 1.0), (False, 5.0)])
@pytest.mark.parametrize("world", [2, 3])
def test_emulated_ranks_vjp_equals_single_call(world, is_warmup, lam):
    """The three-phase VJP over emulated ranks equals dwa_retrieve_bwd on the
    whole pool (rtol 1e-5), key gradients included."""
    from matrix_b200.retrieval import retrieve_backward
    from matrix_b200.sharded import shard_rows
    cfg, x = _case()
    rng = np.random.default_rng(5)
    g_alphas = rng.standard_normal((x.z.shape[0], cfg.k_max)).astype(np.float32)
    g_soft = (rng.standard_normal((x.z.shape[0], cfg.N)) * 50).astype(np.float32)
    shards = shard_rows(x.list_offsets, world)
    got, (a, i, sf) = _emulated_bwd(cfg, x, shards, is_warmup, lam, g_alphas, g_soft)
    max_list = int(np.diff(x.list_offsets).max())
    ref = retrieve_backward(_dev(x.z), _dev(x.W_Q), _dev(x.aspect_weights), torch.tensor(x.tau).cuda(),
                            _dev(x.centroids), _dev(x.keys), lam, is_warmup, a, i, sf, _dev(g_alphas),
                            _dev(g_soft), k=cfg.k_max, m=cfg.m, T=cfg.T, list_offsets=_dev(x.list_offsets),
                            max_list=max_list, want_key_grad=True)
    for name in ("g_z", "g_W_Q", "g_aspect_weights", "g_pool_keys"):
        assert_close(got[name], ref[name].cpu().numpy(), TOL, name=f"{name} world={world}")
    r = float(ref["g_tau"])
    assert abs(float(got["g_tau"]) - r) <= TOL * max(abs(r), 1e-3)


def test_emulated_vjp_with_empty_rank_and_alphas_only():
    """An empty middle rank (zero partials, phase 3 only) and the alphas'
    cotangent alone (phase 2 visits only probed tiles)."""
    from matrix_b200.retrieval import retrieve_backward
    cfg, x = _case(seed=33)
    rng = np.random.default_rng(6)
    g_alphas = rng.standard_normal((x.z.shape[0], cfg.k_max)).astype(np.float32)
    off = x.list_offsets
    mid = int(off[len(off) // 2])
    shards = [(0, mid), (mid, mid), (mid, cfg.N)]
    from matrix_b200.sharded import (bwd_workspace, retrieve_bwd_finish, retrieve_bwd_local1,
                                     retrieve_bwd_local2)
    from matrix_b200.retrieval import retrieve
    z, W_Q, aw = _dev(x.z), _dev(x.W_Q), _dev(x.aspect_weights)
    tau, cents, offd, keys = torch.tensor(x.tau).cuda(), _dev(x.centroids), _dev(off), _dev(x.keys)
    max_list = int(np.diff(off).max())
    kw = dict(k=cfg.k_max, m=cfg.m, T=cfg.T, max_list=max_list)
    a, i, _ = retrieve(z, W_Q, aw, tau, cents, keys, 5.0, False, k=cfg.k_max, m=cfg.m, T=cfg.T,
                       list_offsets=offd, max_list=max_list, want_soft_full=False)
    ga = _dev(g_alphas)
    wss = [bwd_workspace(z, W_Q, hi - lo, C=cfg.C, **kw) for lo, hi in shards]
    locs = [keys[:, lo:hi].contiguous() for lo, hi in shards]
    p1 = sum(retrieve_bwd_local1(wss[r], z, W_Q, aw, tau, cents, locs[r], offd, 5.0, False, i, None, None,
                                 row_lo=lo, n_global=cfg.N, **kw) for r, (lo, hi) in enumerate(shards))
    p2 = sum(retrieve_bwd_local2(wss[r], z, W_Q, aw, tau, cents, locs[r], offd, 5.0, False, a, i, None, ga, None,
                                 p1, row_lo=lo, **kw)[0] for r, (lo, hi) in enumerate(shards))
    got = retrieve_bwd_finish(wss[1], z, W_Q, aw, p2, C=cfg.C, **kw)
    ref = retrieve_backward(z, W_Q, aw, tau, cents, keys, 5.0, False, a, i, None, ga, None, k=cfg.k_max, m=cfg.m,
                            T=cfg.T, list_offsets=offd, max_list=max_list)
    torch.cuda.synchronize()
    for name in ("g_z", "g_W_Q", "g_aspect_weights"):
        assert_close(got[name].cpu().numpy(), ref[name].cpu().numpy(), TOL, name=name)


def _allgather_rank(rank, world, port, out_dir):
    """``PeerAllGather`` against NCCL's all-gather on the same data: eager calls
    back to back (the two buffer halves alternate), then calls captured in a
    CUDA graph and replayed with new inputs."""
    import torch.distributed as dist
    from datetime import timedelta
    from matrix_b200.peer import PeerAllGather
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    pg = None
    try:
        shape = (8, 131)                       # a summary's shape: 8 queries, top-k 64
        pg = PeerAllGather(8 * 131 * 4, dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        ok = []
        for _ in range(5):
            src = torch.randn(shape, generator=g, device=dev)
            got = pg(src)
            ref = torch.empty((world,) + shape, device=dev)
            dist.all_gather_into_tensor(ref, src)
            ok.append(bool(torch.equal(got, ref)))
        src = torch.empty(shape, device=dev)
        out1 = torch.empty((world,) + shape, device=dev)
        out2 = torch.empty((world,) + shape, device=dev)
        src.normal_(generator=g)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            pg(src, out1)                       # warm-up outside the graph
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                pg(src, out1)
                pg(src * 2, out2)
        torch.cuda.current_stream(dev).wait_stream(s)
        for rep in range(3):
            src.normal_(generator=g)
            graph.replay()
            ref = torch.empty((world,) + shape, device=dev)
            dist.all_gather_into_tensor(ref, src)
            ok.append(bool(torch.equal(out1, ref)) and bool(torch.equal(out2, ref * 2)))
        torch.cuda.synchronize(dev)
        del graph
        ok.append(pg.status() == 0)
        np.save(os.path.join(out_dir, f"ag{rank}.npy"), np.array(ok))
    finally:
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_ranks_peer_allgather_equals_nccl(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_allgather_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        ok = np.load(tmp_path / f"ag{rank}.npy")
        assert ok.all(), f"rank {rank}: {ok}"
