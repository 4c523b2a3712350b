"""Row-sharded IVF retrieval over P ranks (one process per GPU).

Replaces the reference's model-sharded retrieval, which turns IVF off and
all-gathers every rank's full-pool scores (src/dwa/retrieval.py:74-79, 121-138)
and then fetches the winners with a masked psum (src/dwa/model.py:16-47).  Here
IVF stays on and only k candidates per query cross the interconnect:

1. ``retrieve_local`` on every rank (``dwa_retrieve_local``): rank p holds the
   keys of pool rows ``[row_lo, row_hi)``; centroids, ``W_Q``, aspect weights,
   ``tau`` and the global CSR ``list_offsets`` are replicated, so every rank
   picks the same top-m lists and scores the part of them it holds.  Output:
   a summary ``[B, 2k+3]`` per rank (see ``summary_width``) and, with
   soft_full, the raw scores of the rank's rows.
2. ``gather_summaries``: one all-gather of ``B*(2k+3)*4`` bytes per rank
   (peer-mapped buffers, ``dwa_peer_allgather``, on an NCCL group).
3. ``retrieve_merge`` on every rank (``dwa_retrieve_merge``): the global top-k
   (ties to the lower pool row), alphas as the single-device call defines
   them, and the rank's soft_full slice normalised with the merged softmax
   statistics.

The result equals ``retrieve`` on the whole pool: indices bit-exact, alphas
and soft_full up to the order in which partial sums are added.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace


def summary_width(k: int) -> int:
    """Floats per query in a rank's summary: k scores, k global rows (int32
    bits), the partial gate sum, the soft_full max and sum of exp."""
    return 2 * k + 3


@dataclass(frozen=True)
class RowShard:
    """This rank's rows ``[row_lo, row_hi)`` of an ``n_global``-row pool and the
    process group of the ranks that hold the other rows (``None``: one rank)."""

    row_lo: int
    row_hi: int
    n_global: int
    group: object = None


def shard_rows(list_offsets, world: int) -> list[tuple[int, int]]:
    """Contiguous row ranges ``[(row_lo, row_hi)] * world`` made of whole lists,
    balanced by rows: rank p's range ends at the list boundary nearest to
    ``(p+1) * N / world``.  ``list_offsets`` is the CSR ``[C+1]`` (any array
    type).  A rank may get no rows when there are fewer lists than ranks."""
    off = np.asarray(list_offsets.cpu() if isinstance(list_offsets, torch.Tensor) else list_offsets,
                     dtype=np.int64)
    if off.ndim != 1 or off.size < 2 or off[0] != 0 or np.any(np.diff(off) < 0):
        raise ValueError("list_offsets must be a non-decreasing CSR array starting at 0")
    if world < 1:
        raise ValueError("world must be >= 1")
    n = int(off[-1])
    bounds = [0]
    for p in range(1, world):
        target = p * n / world
        j = int(np.argmin(np.abs(off - target)))
        bounds.append(max(bounds[-1], int(off[j])))
    bounds.append(n)
    return [(bounds[p], bounds[p + 1]) for p in range(world)]


_peer_gathers: dict = {}


def peer_gather(nbytes: int, device, group=None):
    """The ``PeerAllGather`` of ``nbytes`` per rank for ``group`` on ``device``,
    made on first use (a collective: every rank reaches it at the same call),
    or ``None`` where it does not apply: no NCCL group of two or more ranks, or
    ``DWA_PEER_GATHER=0`` (then the callers use NCCL's all-gather)."""
    import os
    import torch.distributed as dist
    if os.environ.get("DWA_PEER_GATHER", "1") == "0" or nbytes % 16:
        return None
    if not (dist.is_available() and dist.is_initialized()) or dist.get_backend(group) != "nccl":
        return None
    if dist.get_world_size(group) < 2:
        return None
    key = (id(group), int(nbytes), torch.device(device).index)
    pg = _peer_gathers.get(key)
    if pg is None:
        from .peer import PeerAllGather
        pg = _peer_gathers[key] = PeerAllGather(nbytes, device, group)
    return pg


def gather_summaries(summary: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's ``[B, 2k+3]`` summary into ``[P, B, 2k+3]`` (rank
    order).  One exchange: through peer-mapped buffers on an NCCL group
    (``peer_gather``), else one NCCL / gloo all-gather; with no process group,
    the summary alone."""
    import torch.distributed as dist
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return summary.unsqueeze(0)
    world = dist.get_world_size(group)
    if world == 1:
        return summary.unsqueeze(0)
    summary = summary.contiguous()
    pg = peer_gather(summary.numel() * summary.element_size(), summary.device, group)
    if pg is not None:
        return pg(summary)
    out = torch.empty((world,) + tuple(summary.shape), dtype=summary.dtype, device=summary.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, summary, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), summary, group=group)
    return out


def _dims(B, S, d_k, d_A, C, m, k, max_list, N, T, zdt):
    return _lib.RetrieveDims(B, S, d_k, d_A, C, m, k, int(max_list), int(N), float(T), zdt)


def retrieve_local(z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                   is_warmup, *, k, m, T, row_lo, n_global, max_list, use_ivf=True,
                   want_soft_full=True):
    """``dwa_retrieve_local``: this rank's summary ``[B, 2k+3]`` and, with
    ``want_soft_full``, the raw scores ``[B, N_local]`` of its rows."""
    require_cuda("z", z)
    dev = z.device
    require_cuda("local_keys", local_keys, dev)
    if local_keys.dtype != torch.float32 or local_keys.dim() != 3:
        raise ValueError("local_keys must be float32 [S, N_local, d_k]")
    S, n_loc, d_k = local_keys.shape
    B, d_A = z.shape
    C = centroids.shape[1] if use_ivf else 1
    if use_ivf:
        require_cuda("centroids", centroids, dev)
        require_cuda("list_offsets", list_offsets, dev)
        if list_offsets.dtype != torch.int64 or list_offsets.numel() != C + 1:
            raise ValueError("list_offsets must be int64 [C+1] (global rows)")
    lam = lambda_val if isinstance(lambda_val, torch.Tensor) else torch.tensor(
        [float(lambda_val)], dtype=torch.float32, device=dev)
    lam = lam.reshape(1).float().contiguous()
    tau_t = tau.reshape(1).float().contiguous()
    W_Q = W_Q.float().contiguous()
    aw = aspect_weights.float().contiguous()
    dims = _dims(B, S, d_k, d_A, C, m, k, max_list or 0, n_loc, T, dtype_code(z.dtype, "z"))
    shard = _lib.Shard(int(row_lo), int(n_global))
    summary = torch.empty((B, summary_width(k)), dtype=torch.float32, device=dev)
    soft = torch.empty((B, n_loc), dtype=torch.float32, device=dev) if want_soft_full else None
    lib = _lib.load()
    ws, ws_bytes = None, 0
    if n_loc > 0:          # a rank without rows only writes an empty summary
        ws_bytes = lib.dwa_retrieve_workspace_bytes(dims, int(use_ivf), int(want_soft_full))
        if ws_bytes == 0:
            raise _lib.DwaError(f"dwa_retrieve_workspace_bytes: {_lib.last_error()}")
        ws = workspace(dev, "retrieve_local", ws_bytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve_local(stream_of(dev), dims, shard, int(use_ivf), int(bool(is_warmup)),
                                    ptr(lam), ptr(z), ptr(W_Q), ptr(aw), ptr(tau_t),
                                    ptr(centroids) if use_ivf else None,
                                    ptr(list_offsets) if use_ivf else None, ptr(local_keys),
                                    ptr(summary), ptr(soft), ptr(ws), ws_bytes)
    _lib.check(rc, "dwa_retrieve_local")
    return summary, soft


def retrieve_merge(summaries, lambda_val, tau, is_warmup, *, k, T, soft_full=None):
    """``dwa_retrieve_merge``: ``(alphas [B,k], indices [B,k] int32)`` from the
    gathered ``[P, B, 2k+3]`` summaries; ``soft_full`` (this rank's raw slice,
    if given) is normalised in place."""
    require_cuda("summaries", summaries)
    dev = summaries.device
    P, B, W = summaries.shape
    if W != summary_width(k):
        raise ValueError(f"summaries must be [P, B, {summary_width(k)}]")
    lam = lambda_val if isinstance(lambda_val, torch.Tensor) else torch.tensor(
        [float(lambda_val)], dtype=torch.float32, device=dev)
    lam = lam.reshape(1).float().contiguous()
    tau_t = tau.reshape(1).float().contiguous()
    n_soft = 0 if soft_full is None else soft_full.shape[1]
    if soft_full is not None:
        require_cuda("soft_full", soft_full, dev)
        if soft_full.dtype != torch.float32 or soft_full.shape[0] != B or not soft_full.is_contiguous():
            raise ValueError("soft_full must be contiguous float32 [B, N_local]")
    dims = _dims(B, 1, 1, 1, 1, 1, k, 0, n_soft, T, _lib.DWA_F32)
    alphas = torch.empty((B, k), dtype=torch.float32, device=dev)
    indices = torch.empty((B, k), dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, "retrieve_merge", lib.dwa_retrieve_merge_workspace_bytes(dims))
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve_merge(stream_of(dev), dims, P, ptr(summaries.contiguous()),
                                    int(bool(is_warmup)), ptr(lam), ptr(tau_t), ptr(alphas),
                                    ptr(indices), ptr(soft_full), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve_merge")
    return alphas, indices


def sharded_retrieve(z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                     is_warmup, shard: RowShard, *, k, m, T, max_list=None, use_ivf=True,
                     want_soft_full=True):
    """The three steps on this rank: ``(alphas [B,k], indices [B,k] int32,
    soft_full [B, N_local] or None)``; every rank gets the same alphas and
    indices and its own normalised slice of soft_full."""
    if local_keys.shape[1] != shard.row_hi - shard.row_lo:
        raise ValueError("local_keys must hold exactly the rows [row_lo, row_hi)")
    if use_ivf and max_list is None:
        max_list = int((list_offsets[1:] - list_offsets[:-1]).max().item())
    summary, soft = retrieve_local(z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets,
                                   lambda_val, is_warmup, k=k, m=m, T=T, row_lo=shard.row_lo,
                                   n_global=shard.n_global, max_list=max_list or 0, use_ivf=use_ivf,
                                   want_soft_full=want_soft_full)
    gathered = gather_summaries(summary, shard.group)
    alphas, indices = retrieve_merge(gathered, lambda_val, tau, is_warmup, k=k, T=T, soft_full=soft)
    return alphas, indices, soft


# ---------------------------------------------------------------------------
# The retrieval VJP over a row-sharded pool (dwa_retrieve_bwd_local1/2, finish)
# ---------------------------------------------------------------------------

def _bwd_args(z, W_Q, aspect_weights, tau, lambda_val, n_rows, *, k, m, T, C, max_list):
    dev = z.device
    lam = lambda_val if isinstance(lambda_val, torch.Tensor) else torch.tensor(
        [float(lambda_val)], dtype=torch.float32, device=dev)
    B, d_A = z.shape
    S, d_k, _ = W_Q.shape
    dims = _dims(B, S, d_k, d_A, C, m, k, max_list or 0, max(int(n_rows), 1), T, dtype_code(z.dtype, "z"))
    return dims, lam.reshape(1).float().contiguous(), tau.reshape(1).float().contiguous(), \
        W_Q.float().contiguous(), aspect_weights.float().contiguous()


def _bwd_ws_bytes(z, W_Q, n_rows, *, k, m, T, C, max_list, use_ivf):
    dims = _dims(z.shape[0], W_Q.shape[0], W_Q.shape[1], z.shape[1], C, m, k, max_list or 0,
                 max(int(n_rows), 1), T, dtype_code(z.dtype, "z"))
    nbytes = _lib.load().dwa_retrieve_bwd_local_workspace_bytes(dims, int(use_ivf))
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_retrieve_bwd_local_workspace_bytes: {_lib.last_error()}")
    return nbytes


def bwd_workspace(z, W_Q, n_rows, *, k, m, T, C, max_list, use_ivf=True):
    """A workspace for the three phases of one rank's call (one per emulated
    rank when several share a GPU)."""
    return torch.zeros(_bwd_ws_bytes(z, W_Q, n_rows, k=k, m=m, T=T, C=C, max_list=max_list, use_ivf=use_ivf),
                       dtype=torch.uint8, device=z.device)


def retrieve_bwd_local1(ws, z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                        is_warmup, indices, soft_local, g_soft_local, *, k, m, T, row_lo, n_global, max_list,
                        use_ivf=True):
    """Phase 1 on this rank's rows: ``part1 [B, k+3]`` (zeros for a rank without rows)."""
    B = z.shape[0]
    n_loc = local_keys.shape[1]
    part1 = torch.zeros((B, k + 3), dtype=torch.float32, device=z.device)
    if n_loc == 0:
        return part1
    C = centroids.shape[1] if use_ivf else 1
    dims, lam, tau_t, W_Q, aw = _bwd_args(z, W_Q, aspect_weights, tau, lambda_val, n_loc, k=k, m=m, T=T, C=C,
                                          max_list=max_list)
    lib = _lib.load()
    with torch.cuda.device(z.device):
        rc = lib.dwa_retrieve_bwd_local1(
            stream_of(z.device), dims, _lib.Shard(int(row_lo), int(n_global)), int(use_ivf), int(bool(is_warmup)),
            ptr(lam), ptr(z), ptr(W_Q), ptr(aw), ptr(tau_t), ptr(centroids) if use_ivf else None,
            ptr(list_offsets) if use_ivf else None, ptr(local_keys), ptr(indices.int().contiguous()),
            ptr(soft_local), ptr(g_soft_local), ptr(part1), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve_bwd_local1")
    return part1


def retrieve_bwd_local2(ws, z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                        is_warmup, alphas, indices, soft_local, g_alphas, g_soft_local, part1_sum, *, k, m, T,
                        row_lo, max_list, use_ivf=True, want_key_grad=False):
    """Phase 2: ``(part2 [B, S*d_k+1], key gradient of this rank's rows or None)``."""
    B = z.shape[0]
    S, n_loc, d_k = local_keys.shape
    part2 = torch.zeros((B, S * d_k + 1), dtype=torch.float32, device=z.device)
    g_keys = torch.zeros(tuple(local_keys.shape), dtype=torch.float32, device=z.device) if want_key_grad else None
    if n_loc == 0:
        return part2, g_keys
    C = centroids.shape[1] if use_ivf else 1
    dims, lam, tau_t, W_Q, aw = _bwd_args(z, W_Q, aspect_weights, tau, lambda_val, n_loc, k=k, m=m, T=T, C=C,
                                          max_list=max_list)
    lib = _lib.load()
    with torch.cuda.device(z.device):
        rc = lib.dwa_retrieve_bwd_local2(
            stream_of(z.device), dims, _lib.Shard(int(row_lo), 0), int(use_ivf), int(bool(is_warmup)), ptr(lam),
            ptr(tau_t), ptr(aw), ptr(list_offsets) if use_ivf else None, ptr(local_keys),
            ptr(alphas.float().contiguous()) if alphas is not None else None,
            ptr(indices.int().contiguous()) if indices is not None else None, ptr(soft_local),
            ptr(g_alphas.float().contiguous()) if g_alphas is not None else None, ptr(g_soft_local),
            ptr(part1_sum.contiguous()), ptr(part2), ptr(g_keys), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve_bwd_local2")
    return part2, g_keys


def retrieve_bwd_finish(ws, z, W_Q, aspect_weights, part2_sum, *, k, m, T, C, max_list, use_ivf=True):
    """Phase 3: ``dict(g_z, g_W_Q, g_aspect_weights, g_tau)`` from the summed part2."""
    dev = z.device
    f32 = dict(dtype=torch.float32, device=dev)
    dims, _, _, W_Qc, aw = _bwd_args(z, W_Q, aspect_weights, torch.zeros(1, device=dev), 0.0, 1, k=k, m=m, T=T, C=C,
                                     max_list=max_list)
    out = dict(g_z=torch.empty((z.shape[0], z.shape[1]), **f32), g_W_Q=torch.empty(tuple(W_Q.shape), **f32),
               g_aspect_weights=torch.empty((W_Q.shape[0],), **f32), g_tau=torch.empty((), **f32))
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve_bwd_finish(stream_of(dev), dims, int(use_ivf), ptr(z), ptr(W_Qc), ptr(aw),
                                         ptr(part2_sum.contiguous()), ptr(out["g_z"]), ptr(out["g_W_Q"]),
                                         ptr(out["g_aspect_weights"]), ptr(out["g_tau"]), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve_bwd_finish")
    return out


def sharded_retrieve_backward(z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                              is_warmup, shard: RowShard, alphas, indices, soft_local, g_alphas, g_soft_local, *,
                              k, m, T, max_list=None, use_ivf=True, want_key_grad=False):
    """The VJP of ``sharded_retrieve`` on this rank: the three phases with one
    all-reduce of ``[B, k+3]`` and one of ``[B, S*d_k+1]`` floats between them.
    Returns ``dict(g_z, g_W_Q, g_aspect_weights, g_tau, g_pool_keys)`` with the
    key gradient of this rank's rows (or None); every rank gets the same
    parameter gradients."""
    import torch.distributed as dist
    if use_ivf and max_list is None:
        max_list = int((list_offsets[1:] - list_offsets[:-1]).max().item())
    C = centroids.shape[1] if use_ivf else 1
    n_loc = local_keys.shape[1]
    ws = workspace(z.device, "retrieve_bwd_local",
                   _bwd_ws_bytes(z, W_Q, n_loc, k=k, m=m, T=T, C=C, max_list=max_list, use_ivf=use_ivf))
    world = dist.get_world_size(shard.group) if dist.is_available() and dist.is_initialized() else 1
    part1 = retrieve_bwd_local1(ws, z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets, lambda_val,
                                is_warmup, indices, soft_local, g_soft_local, k=k, m=m, T=T, row_lo=shard.row_lo,
                                n_global=shard.n_global, max_list=max_list, use_ivf=use_ivf)
    if world > 1:
        dist.all_reduce(part1, group=shard.group)
    part2, g_keys = retrieve_bwd_local2(ws, z, W_Q, aspect_weights, tau, centroids, local_keys, list_offsets,
                                        lambda_val, is_warmup, alphas, indices, soft_local, g_alphas, g_soft_local,
                                        part1, k=k, m=m, T=T, row_lo=shard.row_lo, max_list=max_list,
                                        use_ivf=use_ivf, want_key_grad=want_key_grad)
    if world > 1:
        dist.all_reduce(part2, group=shard.group)
    out = retrieve_bwd_finish(ws, z, W_Q, aspect_weights, part2, k=k, m=m, T=T, C=C, max_list=max_list,
                              use_ivf=use_ivf)
    out["g_pool_keys"] = g_keys
    return out
