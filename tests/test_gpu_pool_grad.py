"""Pool-row gradient scatter (``dwa_pool_grad_scatter``), the VJP of the gather
``pool[indices]`` (model.py:193-195), against ``np.add.at`` in float64:
duplicates across queries, f32 and bf16 gradient buffers, a row window (one
rank's rows), bit-identical repeats, the assembly backward's g_rows end to end,
several emulated ranks, and an out-of-range row (status bit, row skipped)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _case(n_rows=5000, D=1088, B=8, k=32, seed=0):
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, n_rows, size=(B, k)).astype(np.int32)
    idx[1, :5] = idx[0, :5]                  # the same rows chosen by two queries
    idx[2, 7] = idx[0, 0]
    g = rng.standard_normal((B, k, D), dtype=np.float32)
    base = rng.standard_normal((n_rows, D), dtype=np.float32)
    return idx, g, base


def _ref(base, idx, g, lo=0, hi=None):
    hi = base.shape[0] if hi is None else hi
    out = base.astype(np.float64)
    flat_i, flat_g = idx.reshape(-1), g.reshape(-1, g.shape[-1]).astype(np.float64)
    keep = (flat_i >= lo) & (flat_i < hi)
    np.add.at(out, flat_i[keep], flat_g[keep])
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scatter_matches_add_at(dtype):
    from matrix_b200.pool_grad import scatter_pool_grad
    from matrix_b200.runtime import raise_on_device_status
    idx, g, base = _case()
    if dtype == torch.bfloat16:
        base = torch.from_numpy(base).bfloat16().float().numpy()
    gp = torch.from_numpy(base).cuda().to(dtype)
    scatter_pool_grad(torch.from_numpy(g).cuda(), torch.from_numpy(idx).cuda(), gp)
    torch.cuda.synchronize()
    assert_close(gp.float().cpu().numpy(), _ref(base, idx, g), 1e-6 if dtype == torch.float32 else 1e-2,
                 name=f"g_pool {dtype}")
    raise_on_device_status()


def test_window_and_determinism():
    from matrix_b200.pool_grad import scatter_pool_grad
    idx, g, base = _case()
    lo, hi = 1200, 3700
    outs = []
    for _ in range(2):
        gp = torch.from_numpy(base[lo:hi].copy()).cuda()
        scatter_pool_grad(torch.from_numpy(g).cuda(), torch.from_numpy(idx).cuda(), gp, row_lo=lo,
                          n_global=base.shape[0])
        outs.append(gp.cpu().numpy())
    np.testing.assert_array_equal(outs[0], outs[1])
    assert_close(outs[0], _ref(base, idx, g, lo, hi)[lo:hi], 1e-6, name="window")


def test_emulated_ranks_cover_the_pool():
    """Each rank scatters every rank's contributions into its own rows; together
    they equal the single-device scatter."""
    from matrix_b200.pool_grad import scatter_pool_grad
    idx, g, base = _case(seed=3)
    parts = []
    bounds = [0, 1700, 1700, 5000]          # an empty middle rank
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        gp = torch.from_numpy(base[lo:hi].copy()).cuda()
        if hi > lo:
            scatter_pool_grad(torch.from_numpy(g).cuda(), torch.from_numpy(idx).cuda(), gp, row_lo=lo,
                              n_global=base.shape[0])
        parts.append(gp.cpu().numpy())
    assert_close(np.concatenate(parts), _ref(base, idx, g), 1e-6, name="ranks")


def test_assembly_backward_rows_scatter_like_autodiff():
    """g_pool of the gather = scatter of the assembly backward's g_rows."""
    from matrix_b200.assembly import assemble_backward, assemble_forward
    from matrix_b200.pool_grad import scatter_pool_grad
    from oracle import dwa_oracle as O
    from test_gpu_assembly import _dev, _setup
    cfg, x, idx, alphas = _setup("f32_ragged")
    f = np.float64
    pool = _dev(x.pool)
    h_mid, W, W_act = assemble_forward(pool, _dev(alphas), _dev(x.h_A), _dev(x.W_base), _dev(x.b_base),
                                       torch.tensor(x.gamma).cuda(), cfg.d_B, cfg.r, cfg.d_A,
                                       row_index=_dev(idx))
    grads = assemble_backward(pool, _dev(alphas), _dev(x.h_A), W_act, torch.tensor(x.gamma).cuda(),
                              _dev(x.g_hmid), _dev(x.g_W), cfg.d_B, cfg.r, cfg.d_A, row_index=_dev(idx))
    g_rows = grads[0]
    gp = torch.zeros_like(pool)
    scatter_pool_grad(g_rows, _dev(idx), gp)
    gathered = x.pool[idx].astype(f)
    Wr = O.assemble(gathered, alphas.astype(f), x.h_A.astype(f), x.W_base.astype(f), x.b_base.astype(f),
                    f(x.gamma), cfg.d_B, cfg.r, cfg.d_A)[1]
    rg = O.assemble_bwd(gathered, alphas.astype(f), x.h_A.astype(f), Wr, f(x.gamma), x.g_hmid.astype(f),
                        x.g_W.astype(f), cfg.d_B, cfg.r, cfg.d_A)[0]
    ref = np.zeros(x.pool.shape, f)
    np.add.at(ref, idx.reshape(-1), rg.reshape(-1, rg.shape[-1]))
    assert_close(gp.cpu().numpy(), ref, 1e-5, name="g_pool")


def test_out_of_range_row_sets_status_and_is_skipped():
    from matrix_b200.pool_grad import scatter_pool_grad
    from matrix_b200.runtime import workspace_status
    idx, g, base = _case()
    idx[3, 4] = base.shape[0] + 7
    workspace_status(clear=True)
    gp = torch.from_numpy(base.copy()).cuda()
    scatter_pool_grad(torch.from_numpy(g).cuda(), torch.from_numpy(idx).cuda(), gp)
    st = workspace_status(clear=True)
    assert any(v & 0x1 for v in st.values())
    keep = idx.copy()
    keep[3, 4] = -1
    ref = base.astype(np.float64)
    m = keep.reshape(-1) >= 0
    np.add.at(ref, keep.reshape(-1)[m], g.reshape(-1, g.shape[-1])[m].astype(np.float64))
    assert_close(gp.cpu().numpy(), ref, 1e-6, name="skipped")


def _bf16(x):
    from matrix_b200.synthetic import bf16_round
    return bf16_round(np.asarray(x, np.float32))


@pytest.mark.parametrize("bounds", [[0, 5000], [0, 1700, 1700, 5000], [0, 900, 2600, 4100, 5000]])
def test_owner_exchange_equals_sorted_scatter(bounds):
    """Emulated ranks on one GPU return their rows' gradients to the owners
    through receive areas (dwa_pool_grad_send: bf16 rows, pad slots
    elsewhere; then each owner's dwa_pool_grad_scatter_typed).  Every owner's
    rows equal np.add.at of the bf16-rounded contributions in float64 (rtol
    1e-5 on the f32 sums); a second call into the other areas with fewer
    contributions adds only those (the pad slots of the earlier call are
    not replayed); no status bit is set by the pad slots."""
    from matrix_b200.pool_grad import PoolGradExchange
    from matrix_b200.runtime import raise_on_device_status
    world = len(bounds) - 1
    idx, g, _ = _case(seed=9)
    D = g.shape[-1]
    per = idx.shape[0] // world if world > 1 else idx.shape[0]
    sends = [(idx[r * per:(r + 1) * per], g[r * per:(r + 1) * per]) for r in range(world)]
    slot = per * idx.shape[1]
    nbytes = PoolGradExchange.area_size(world, slot, D)
    areas = [[torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(world)] for _ in range(2)]
    ex = [PoolGradExchange.from_areas(world, r, bounds, slot, D, areas) for r in range(world)]
    pools = [torch.zeros((bounds[r + 1] - bounds[r], D), dtype=torch.float32, device="cuda") for r in range(world)]
    n_global = bounds[-1]
    expect = np.zeros((n_global, D))
    for call, take in enumerate((slot, slot // 3)):
        parity = call & 1
        for r in range(world):
            i_r, g_r = sends[r]
            i_r, g_r = i_r.reshape(-1)[:take], g_r.reshape(-1, D)[:take]
            ex[r].send(torch.from_numpy(g_r).cuda(), torch.from_numpy(i_r).cuda(), parity)
            np.add.at(expect, i_r, _bf16(g_r).astype(np.float64))
        for r in range(world):
            ex[r].scatter(pools[r], parity)
        torch.cuda.synchronize()
        got = np.concatenate([p.cpu().numpy() for p in pools])
        assert_close(got, expect, 1e-5, name=f"call {call}")
    raise_on_device_status()
