"""Pool-row gradients: the VJP of the gather ``pool[indices]``.

The reference gathers the winning pool rows with ``pool_vecs[indices]``
(src/dwa/model.py:193-195; ``_distributed_gather``, model.py:16-47, when the
pool is sharded) and lets autodiff form the dense ``[N, D]`` pool gradient.
Only ``B*k`` rows are non-zero, so here the backward's ``g_rows [B, k, D]``
are scattered into the selected rows (``dwa_pool_grad_scatter``: sorted,
deterministic, no atomics):

* ``scatter_pool_grad``: one device, into ``g_pool [N, D]`` (or one rank's rows).
* ``PoolGradExchange``: a row-sharded pool over several ranks.  Each rank
  stores its contributions, as bf16 rows, straight into the receive area of
  the rank that owns each row (``dwa_pool_grad_send``, peer stores over
  NVLink: ``B*k*D*2`` bytes leave a rank), one small collective orders the
  stores before the reads, and every owner scatters its own area.
* ``scatter_pool_grad_gathered``: several ranks, by all-gather.  Every rank all-gathers the
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


class PoolGradExchange:
    """Receive areas for returning row gradients to their owners.

    ``row_bounds``: the ``world + 1`` global row boundaries of the row-sharded
    pool; ``slot``: the most contributions one rank sends per call (its
    ``B_p * k``).  Every rank allocates two areas (used alternately, so a rank
    one call ahead never writes into an area its owner still reads) and maps
    every other rank's by CUDA IPC.  Collective: every rank of ``group``
    constructs it at the same point.  ``from_areas`` builds the same object for
    ranks emulated on one GPU (every area local)."""

    def __init__(self, row_bounds, slot: int, D: int, device, group=None, rows_dtype=torch.bfloat16):
        import torch.distributed as dist
        from .peer import map_peer_buffers
        world = dist.get_world_size(group)
        self._init(world, dist.get_rank(group), row_bounds, slot, D, device, rows_dtype, group)
        self.areas = [torch.zeros(self.area_bytes, dtype=torch.uint8, device=device) for _ in range(2)]
        self._bases, self._opened = [], []
        for a in self.areas:
            b, o = map_peer_buffers(a, group)
            self._bases.append(b)
            self._opened += o

    @classmethod
    def from_areas(cls, world, rank, row_bounds, slot, D, areas_by_rank, rows_dtype=torch.bfloat16):
        """Rank ``rank`` of ``world`` ranks emulated on one GPU:
        ``areas_by_rank[parity][r]`` is rank r's area (each ``area_bytes``)."""
        self = cls.__new__(cls)
        self._init(world, rank, row_bounds, slot, D, areas_by_rank[0][rank].device, rows_dtype, None)
        self.areas = [areas_by_rank[0][rank], areas_by_rank[1][rank]]
        self._bases = [[t.data_ptr() for t in areas_by_rank[p]] for p in range(2)]
        self._opened = []
        return self

    @staticmethod
    def area_size(world, slot, D, rows_dtype=torch.bfloat16) -> int:
        return int(_lib.load().dwa_pool_grad_recv_bytes(world, slot, D, dtype_code(rows_dtype, "rows")))

    def _init(self, world, rank, row_bounds, slot, D, device, rows_dtype, group):
        import ctypes as C
        self.world, self.rank, self.slot, self.D = int(world), int(rank), int(slot), int(D)
        self.device, self.group, self.rows_dtype = device, group, rows_dtype
        self.bounds = [int(b) for b in row_bounds]
        if len(self.bounds) != self.world + 1:
            raise ValueError("row_bounds needs world + 1 entries")
        self.area_bytes = self.area_size(self.world, self.slot, self.D, rows_dtype)
        if self.area_bytes == 0:
            raise _lib.DwaError(f"dwa_pool_grad_recv_bytes: world {world}, slot {slot}, D {D} not supported")
        self._row_lo = (C.c_int64 * (self.world + 1))(*self.bounds)
        self.parity = 0

    def _shards(self, parity):
        import ctypes as C
        bases = (C.c_void_p * self.world)(*self._bases[parity])
        return bases, _lib.PoolShards(self.world, bases, self._row_lo)

    def send(self, g_rows: torch.Tensor, indices: torch.Tensor, parity: int) -> None:
        """This rank's contributions into their owners' areas of ``parity``."""
        import ctypes as C
        require_cuda("g_rows", g_rows, self.device)
        gr = g_rows.reshape(-1, self.D).float().contiguous()
        idx = indices.reshape(-1).to(torch.int32).contiguous()
        n = idx.numel()
        if gr.shape[0] != n or n > self.slot:
            raise ValueError(f"one index per row and at most slot={self.slot} rows")
        bases, shards = self._shards(parity)
        lib = _lib.load()
        ws = workspace(self.device, "pool_grad_send", 256)
        with torch.cuda.device(self.device):
            rc = lib.dwa_pool_grad_send(stream_of(self.device), self.rank, n, self.slot, self.D, ptr(idx), ptr(gr),
                                        dtype_code(self.rows_dtype, "rows"), C.byref(shards), ptr(ws), ws.numel())
        _lib.check(rc, "dwa_pool_grad_send")

    def scatter(self, g_pool: torch.Tensor, parity: int) -> torch.Tensor:
        """This rank's area of ``parity`` into its rows of ``g_pool``."""
        area = self.areas[parity]
        n = self.world * self.slot
        idx = area[: n * 4].view(torch.int32)
        rows_off = (n * 4 + 255) // 256 * 256
        lo, hi = self.bounds[self.rank], self.bounds[self.rank + 1]
        if g_pool.shape[0] != hi - lo or g_pool.shape[1] != self.D or not g_pool.is_contiguous():
            raise ValueError("g_pool must be this rank's contiguous [rows, D]")
        lib = _lib.load()
        ws = workspace(self.device, "pool_grad", lib.dwa_pool_grad_scatter_workspace_bytes(n))
        with torch.cuda.device(self.device):
            rc = lib.dwa_pool_grad_scatter_typed(
                stream_of(self.device), n, self.D, ptr(idx), dtype_code(self.rows_dtype, "rows"),
                ptr(area[rows_off:]), int(self.bounds[-1]), int(lo), int(hi), dtype_code(g_pool.dtype, "g_pool"),
                ptr(g_pool), ptr(ws), ws.numel())
        _lib.check(rc, "dwa_pool_grad_scatter_typed")
        return g_pool

    def __call__(self, g_rows: torch.Tensor, indices: torch.Tensor, g_pool: torch.Tensor) -> torch.Tensor:
        """Send, order the stores before the reads with one collective, scatter."""
        import torch.distributed as dist
        parity = self.parity
        self.parity ^= 1
        self.send(g_rows, indices, parity)
        if self.world > 1:
            flag = torch.zeros(1, dtype=torch.float32, device=self.device)
            dist.all_reduce(flag, group=self.group)
        return self.scatter(g_pool, parity)

    def close(self) -> None:
        from .peer import close_peer_buffers
        close_peer_buffers(self.device, self._opened)
        self._opened = []
