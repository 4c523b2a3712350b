"""Gather of pool rows from a row-sharded pool (``dwa_gather_rows``,
``PeerPool``), the B200 replacement of ``_distributed_gather``
(src/dwa/model.py:16-47).

One process here (shards emulated on one GPU, the same kernel): uneven shards
with an empty one, rows on every boundary, bf16 and f32 rows, an out-of-range
row (status bit, zero row), and the assembly fed by gathered rows equal to the
assembly reading the whole pool by index.  The two-rank IPC form runs in
``tests/test_gpu_sharded.py``.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _pool(N=3000, D=1088, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((N, D), generator=g).to(dtype).cuda()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gather_from_emulated_shards(dtype):
    from matrix_b200.peer import PeerPool
    pool = _pool(dtype=dtype)
    bounds = [0, 700, 700, 2100, 3000]          # rank 1 holds no rows
    shards = [pool[lo:hi].clone() for lo, hi in zip(bounds[:-1], bounds[1:])]
    pp = PeerPool.from_shards(shards, bounds)
    rng = np.random.default_rng(1)
    idx = rng.integers(0, 3000, size=(7, 33)).astype(np.int32)
    idx[0, :6] = [0, 699, 700, 2099, 2100, 2999]
    got = pp.gather(torch.from_numpy(idx).cuda())
    torch.cuda.synchronize()
    assert got.shape == (7, 33, pool.shape[1]) and got.dtype == dtype
    assert torch.equal(got, pool[torch.from_numpy(idx).long().cuda()])


def test_out_of_range_row_sets_status_and_zeroes():
    from matrix_b200.peer import PeerPool
    from matrix_b200.runtime import workspace_status
    pool = _pool()
    bounds = [0, 1500, 3000]
    pp = PeerPool.from_shards([pool[:1500].clone(), pool[1500:].clone()], bounds)
    workspace_status(clear=True)
    idx = torch.tensor([5, 3000, 2999], dtype=torch.int32).cuda()
    got = pp.gather(idx)
    st = workspace_status(clear=True)
    assert any(v & 0x1 for v in st.values())
    assert torch.equal(got[0], pool[5]) and torch.equal(got[2], pool[2999])
    assert not got[1].float().abs().any()


def test_assembly_on_gathered_rows_equals_index_read():
    """assemble_forward(rows gathered from shards) == assemble_forward(pool,
    row_index=indices): the assembly of a rank's sequences reads the same rows."""
    from matrix_b200.assembly import assemble_forward
    from matrix_b200.peer import PeerPool
    from test_gpu_assembly import _dev, _setup
    cfg, x, idx, alphas = _setup("bf16_small_like")
    pool = _dev(x.pool, torch.bfloat16)
    N = pool.shape[0]
    bounds = [0, N // 3, N // 3, N]
    pp = PeerPool.from_shards([pool[lo:hi].clone() for lo, hi in zip(bounds[:-1], bounds[1:])], bounds)
    args = (_dev(alphas), _dev(x.h_A, torch.bfloat16), _dev(x.W_base), _dev(x.b_base),
            torch.tensor(x.gamma).cuda(), cfg.d_B, cfg.r, cfg.d_A)
    rows = pp.gather(_dev(idx))
    h1, W1, _ = assemble_forward(rows, *args)
    h2, W2, _ = assemble_forward(pool, *args, row_index=_dev(idx))
    torch.cuda.synchronize()
    assert torch.equal(h1, h2) and torch.equal(W1, W2)
