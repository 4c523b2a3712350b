"""Peer access to a row-sharded pool (one process per GPU on one node).

Replaces ``_distributed_gather`` (src/dwa/model.py:16-47), which gathers the
retrieved rows of a model-sharded pool with a masked ``psum`` of ``B*k*D``
values over the model axis.  Here every rank maps the other ranks' pool shards
into its address space once (CUDA IPC handles exchanged over the process
group) and ``PeerPool.gather`` reads each winning row straight from the rank
that holds it (``dwa_gather_rows``: 16-byte loads, over NVLink for peers'
rows).  The gathered rows feed the assembly of this rank's own sequences
(``assemble_forward(rows, ...)``); the backward returns the rows' gradients to
their owners with ``pool_grad.scatter_pool_grad_gathered``.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace


def map_peer_buffers(local: torch.Tensor, group=None):
    """Every rank's ``local`` buffer, readable and writable from this GPU:
    ``(bases, opened)`` with ``bases[r]`` the device address of rank r's buffer
    here (this rank's own for r == rank) and ``opened`` the mappings to close.
    Collective: every rank of ``group`` calls it at the same point with
    buffers of the same size."""
    import torch.distributed as dist
    require_cuda("local", local)
    lib = _lib.load()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    handle = (C.c_char * lib.dwa_ipc_handle_bytes())()
    off = C.c_int64()
    with torch.cuda.device(local.device):
        _lib.check(lib.dwa_ipc_handle(ptr(local), handle, C.byref(off)), "dwa_ipc_handle")
    mine = (bytes(handle), off.value, int(local.numel() * local.element_size()))
    every = [None] * world
    dist.all_gather_object(every, mine, group=group)
    if any(e[2] != mine[2] for e in every):
        raise ValueError("every rank's buffer needs the same size")
    bases, opened = [], []
    with torch.cuda.device(local.device):
        for r, (h, o, _) in enumerate(every):
            if r == rank:
                bases.append(local.data_ptr())
                continue
            p = C.c_void_p()
            _lib.check(lib.dwa_ipc_open(h, o, C.byref(p)), "dwa_ipc_open")
            opened.append((p.value, o))
            bases.append(p.value)
    return bases, opened


def close_peer_buffers(device, opened) -> None:
    lib = _lib.load()
    with torch.cuda.device(device):
        torch.cuda.synchronize(device)
        for p, o in opened:
            _lib.check(lib.dwa_ipc_close(C.c_void_p(p), o), "dwa_ipc_close")


class PeerPool:
    """Every rank's pool rows, readable from this GPU.

    ``local_rows [rows_p, D]`` is this rank's shard (a CUDA tensor that stays
    alive and in place while the pool is used) and ``row_bounds`` the
    ``world + 1`` global row boundaries (rank r holds
    ``[row_bounds[r], row_bounds[r+1])``).  Collective: every rank of ``group``
    constructs its ``PeerPool`` at the same point."""

    def __init__(self, local_rows: torch.Tensor, row_bounds, group=None):
        import torch.distributed as dist
        require_cuda("local_rows", local_rows)
        if local_rows.dim() != 2 or not local_rows.is_contiguous():
            raise ValueError("local_rows must be a contiguous [rows, D] tensor")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        bounds = [int(b) for b in row_bounds]
        if len(bounds) != self.world + 1:
            raise ValueError("row_bounds needs world + 1 entries")
        if bounds[self.rank + 1] - bounds[self.rank] != local_rows.shape[0]:
            raise ValueError("local_rows does not match this rank's row range")
        lib = _lib.load()
        handle = (C.c_char * lib.dwa_ipc_handle_bytes())()
        off = C.c_int64()
        with torch.cuda.device(local_rows.device):
            _lib.check(lib.dwa_ipc_handle(ptr(local_rows), handle, C.byref(off)), "dwa_ipc_handle")
        mine = (bytes(handle), off.value, int(local_rows.shape[1]), str(local_rows.dtype))
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        if any(e[2:] != mine[2:] for e in every):
            raise ValueError("every rank's shard needs the same row width and dtype")
        self._opened = []
        bases = []
        with torch.cuda.device(local_rows.device):
            for r, (h, o, _, _) in enumerate(every):
                if r == self.rank:
                    bases.append(local_rows.data_ptr())
                    continue
                p = C.c_void_p()
                _lib.check(lib.dwa_ipc_open(h, o, C.byref(p)), "dwa_ipc_open")
                self._opened.append((p.value, o))
                bases.append(p.value)
        self._setup(local_rows, bases, bounds)

    @classmethod
    def from_shards(cls, shards, row_bounds):
        """All shards on this GPU (no IPC): the same gather, for one process."""
        self = cls.__new__(cls)
        self.world, self.rank, self._opened = len(shards), 0, []
        self._keep = list(shards)
        self._setup(shards[0], [t.data_ptr() for t in shards], [int(b) for b in row_bounds])
        return self

    def _setup(self, ref, bases, bounds):
        self.device, self.dtype, self.D = ref.device, ref.dtype, int(ref.shape[1])
        self.n_global = bounds[-1]
        self._local = ref
        self._bases = (C.c_void_p * len(bases))(*bases)
        self._row_lo = (C.c_int64 * len(bounds))(*bounds)
        self._shards = _lib.PoolShards(len(bases), self._bases, self._row_lo)

    def gather(self, indices: torch.Tensor) -> torch.Tensor:
        """Rows ``pool[indices]`` (global row numbers, any shape) as a new tensor
        ``indices.shape + (D,)`` in the pool dtype."""
        require_cuda("indices", indices, self.device)
        idx = indices.to(torch.int32).contiguous()
        out = torch.empty(tuple(idx.shape) + (self.D,), dtype=self.dtype, device=self.device)
        lib = _lib.load()
        ws = workspace(self.device, "gather_rows", lib.dwa_gather_rows_workspace_bytes())
        with torch.cuda.device(self.device):
            rc = lib.dwa_gather_rows(stream_of(self.device), idx.numel(), self.D, dtype_code(self.dtype, "pool"),
                                     ptr(idx), C.byref(self._shards), ptr(out), ptr(ws), ws.numel())
        _lib.check(rc, "dwa_gather_rows")
        return out

    def close(self) -> None:
        """Unmap the peers' shards (after every use of them has completed)."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p, o in self._opened:
                _lib.check(lib.dwa_ipc_close(C.c_void_p(p), o), "dwa_ipc_close")
        self._opened = []


class PeerAllGather:
    """All-gather of ``nbytes`` per rank through exchange buffers mapped on
    every GPU of the group (``dwa_peer_allgather``): for the few-kilobyte
    exchanges of a row-sharded step, whose NCCL all-gather costs tens of
    microseconds each.  ``__call__(src)`` returns ``out`` ``[world, *src.shape]``
    in rank order, the same values ``dist.all_gather_into_tensor`` gives.

    Collective: every rank of ``group`` constructs it at the same point, and
    every rank makes the same sequence of calls.  The ranks must be on
    distinct GPUs (a rank waits, bounded, for its peers' data)."""

    def __init__(self, nbytes: int, device, group=None):
        import torch.distributed as dist
        lib = _lib.load()
        self.world, self.rank, self.nbytes = dist.get_world_size(group), dist.get_rank(group), int(nbytes)
        if self.nbytes <= 0 or self.nbytes % 16:
            raise ValueError("nbytes must be a positive multiple of 16")
        size = int(lib.dwa_peer_allgather_buffer_bytes(self.world, self.nbytes))
        if size == 0:
            raise ValueError(f"dwa_peer_allgather supports 1..16 ranks, not {self.world}")
        self.device = torch.device(device)
        self.buffer = torch.zeros(size, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)      # zeroed before any peer writes into it
        bases, self._opened = map_peer_buffers(self.buffer, group)
        self._bases = (C.c_void_p * self.world)(*bases)
        dist.barrier(group)                      # every rank's buffer is mapped and zero

    def __call__(self, src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        require_cuda("src", src)
        if src.numel() * src.element_size() != self.nbytes or not src.is_contiguous():
            raise ValueError(f"src must be a contiguous tensor of {self.nbytes} bytes")
        if out is None:
            out = torch.empty((self.world,) + tuple(src.shape), dtype=src.dtype, device=src.device)
        lib = _lib.load()
        _lib.check(lib.dwa_peer_allgather(stream_of(src.device), self.rank, self.world, ptr(src), self.nbytes,
                                          self._bases, ptr(out)), "dwa_peer_allgather")
        return out

    def status(self, clear: bool = True) -> int:
        """The buffer's status bits (DWA_STATUS_WAIT_TIMEOUT when a wait gave
        up); synchronises the current stream."""
        s = C.c_uint32()
        _lib.check(_lib.load().dwa_peer_allgather_status(stream_of(self.device), ptr(self.buffer), C.byref(s),
                                                          int(clear)), "dwa_peer_allgather_status")
        return int(s.value)

    def close(self) -> None:
        if self._opened:
            close_peer_buffers(self.device, self._opened)
            self._opened = []
