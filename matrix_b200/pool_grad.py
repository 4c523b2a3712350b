"""Pool-row gradients: the VJP of the gather ``pool[indices]``.

The reference gathers the winning pool rows with ``pool_vecs[indices]``
(src/dwa/model.py:193-195; ``_distributed_gather``, model.py:16-47, when the
pool is sharded) and lets autodiff form the dense ``[N, D]`` pool gradient.
Only ``B*k`` rows are non-zero, so here the backward's ``g_rows [B, k, D]``
are scattered into the selected rows (``dwa_pool_grad_scatter``: sorted,
deterministic, no atomics):

* ``scatter_pool_grad``: one device, into ``g_pool [N, D]`` (or one rank's rows).
* ``scatter_pool_grad_gathered``: several ranks.  Every rank all-gathers the
  ``(indices, g_rows)`` of all ranks (``P*B*k*(D+1)*4`` bytes, fixed size, no host
  synchronisation) and scatters the rows it holds: with replicated pools
  (data parallel) every replica applies the same sparse update instead of an
  all-reduce of the dense ``[N, D]`` gradient; with a row-sharded pool each
  rank updates its own rows.
"""

from __future__ import annotations

import torch

from . import _lib
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace

SCATTER_MAX_N = 8192   # contributions one dwa_pool_grad_scatter call accepts


def scatter_pool_grad(g_rows: torch.Tensor, indices: torch.Tensor, g_pool: torch.Tensor, *,
                      row_lo: int = 0, n_global: int | None = None) -> torch.Tensor:
    """``g_pool[row - row_lo] += sum of g_rows[i]`` over ``indices[i] == row`` for the
    rows ``[row_lo, row_lo + g_pool.shape[0])``; returns ``g_pool``."""
    require_cuda("g_rows", g_rows)
    dev = g_rows.device
    require_cuda("indices", indices, dev)
    require_cuda("g_pool", g_pool, dev)
    D = g_rows.shape[-1]
    gr = g_rows.reshape(-1, D).float().contiguous()
    idx = indices.reshape(-1).to(torch.int32).contiguous()
    if idx.numel() != gr.shape[0]:
        raise ValueError("one index per gradient row")
    if g_pool.dim() != 2 or g_pool.shape[1] != D or not g_pool.is_contiguous():
        raise ValueError("g_pool must be contiguous [rows, D]")
    n_rows = g_pool.shape[0]
    n_global = row_lo + n_rows if n_global is None else n_global
    lib = _lib.load()
    n = idx.numel()
    # one call sorts at most SCATTER_MAX_N contributions; larger batches go in
    # consecutive calls (each a deterministic sorted scatter-add, in order)
    chunk = min(n, SCATTER_MAX_N)
    ws = workspace(dev, "pool_grad", lib.dwa_pool_grad_scatter_workspace_bytes(max(chunk, 1)))
    with torch.cuda.device(dev):
        for i0 in range(0, n, SCATTER_MAX_N):
            c = min(SCATTER_MAX_N, n - i0)
            rc = lib.dwa_pool_grad_scatter(stream_of(dev), c, D, ptr(idx[i0:]), ptr(gr[i0:]), int(n_global),
                                           int(row_lo), int(row_lo + n_rows), dtype_code(g_pool.dtype, "g_pool"),
                                           ptr(g_pool), ptr(ws), ws.numel())
            _lib.check(rc, "dwa_pool_grad_scatter")
    return g_pool


def scatter_pool_grad_gathered(g_rows: torch.Tensor, indices: torch.Tensor, g_pool: torch.Tensor, *,
                               row_lo: int, n_global: int, group=None) -> torch.Tensor:
    """All-gather every rank's ``(indices, g_rows)`` and scatter the rows this rank
    holds (``[row_lo, row_lo + g_pool.shape[0])``; the whole pool for replicas)."""
    import torch.distributed as dist
    D = g_rows.shape[-1]
    gr = g_rows.reshape(-1, D).float().contiguous()
    idx = indices.reshape(-1).to(torch.int32).contiguous()
    world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    if world > 1:
        all_gr = torch.empty((world,) + tuple(gr.shape), dtype=gr.dtype, device=gr.device)
        all_idx = torch.empty((world,) + tuple(idx.shape), dtype=idx.dtype, device=idx.device)
        dist.all_gather_into_tensor(all_gr, gr, group=group)
        dist.all_gather_into_tensor(all_idx, idx, group=group)
        gr, idx = all_gr.reshape(-1, D), all_idx.reshape(-1)
    return scatter_pool_grad(gr, idx, g_pool, row_lo=row_lo, n_global=n_global)
