"""DWA assembly with its custom VJP, on libdwa's B200 kernels.

Drop-in for the reference's ``src/dwa/assembly_pallas.py``:

* :func:`pallas_assemble` keeps the signature and the custom-VJP contract of
  ``pallas_assemble`` (assembly_pallas.py:193-222, 332): primal
  ``(h_mid [B,T,d_B], W [B,d_B,d_A])``, ``d_B, r, d_A`` non-differentiable,
  gradients for ``(gathered, alphas, h_A, W_base, b_base, gamma)`` equal to
  ``_pallas_assemble_bwd`` (:246-329).  The VJP is a ``torch.autograd.Function``.
* :func:`shard_pallas_assemble` is the batch-sharded form (:339-385): every rank
  runs its local batch slice; gradients of the replicated ``W_base``, ``b_base``
  and ``gamma`` are summed over the process group in the backward pass.
* :func:`assemble_forward` / :func:`assemble_backward` expose the two C-ABI
  calls directly, including the fused-gather form that reads pool rows by index
  instead of a materialised ``gathered`` tensor (model.py:184-195);
  :func:`assemble_apply` is the h_mid-only call (no W) for generation.

Nothing here computes on the CPU: every entry point requires CUDA tensors and
the built library.
"""

from __future__ import annotations

import torch

from . import _lib
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace


def _dims(B, T, k, D, d_A, d_B, r, act, rows, n_rows):
    return _lib.AssembleDims(B, T, k, D, d_A, d_B, r, act, rows, 0, n_rows)


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.float32 and t.is_contiguous() else t.float().contiguous()


def _check_common(rows, alphas, h_A, d_B, r, d_A, row_index):
    require_cuda("h_A", h_A)
    dev = h_A.device
    require_cuda("rows", rows, dev)
    if h_A.dim() != 3 or h_A.shape[2] != d_A:
        raise ValueError(f"h_A must be [B, T, d_A={d_A}], got {tuple(h_A.shape)}")
    B, T, _ = h_A.shape
    if row_index is None:
        if rows.dim() != 3 or rows.shape[0] != B:
            raise ValueError(f"gathered must be [B={B}, k, D], got {tuple(rows.shape)}")
        k, D, n_rows = rows.shape[1], rows.shape[2], B * rows.shape[1]
    else:
        require_cuda("row_index", row_index, dev)
        if row_index.dtype != torch.int32 or row_index.dim() != 2 or row_index.shape[0] != B:
            raise ValueError("row_index must be int32 [B, k]")
        if rows.dim() != 2:
            raise ValueError("pool must be [N, D]")
        k, D, n_rows = row_index.shape[1], rows.shape[1], rows.shape[0]
    if tuple(alphas.shape) != (B, k):
        raise ValueError(f"alphas must be [B={B}, k={k}], got {tuple(alphas.shape)}")
    if d_A != d_B:
        raise ValueError("d_A must equal d_B for the residual connection")
    if D < d_B * r + r * d_A + d_B:
        raise ValueError(f"D={D} < d_B*r + r*d_A + d_B")
    return dev, B, T, k, D, n_rows


def assemble_forward(rows, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A, *,
                     row_index=None, want_W=True):
    """One ``dwa_assemble_fwd`` call.

    ``rows`` is ``gathered [B,k,D]`` (``row_index=None``) or the pool ``[N,D]``
    with ``row_index [B,k] int32``.  Returns ``(h_mid, W, W_act)``: ``W`` float32
    ``[B,d_B,d_A]`` (``None`` if not wanted) and ``W_act`` the same matrix in
    ``h_A``'s dtype (the backward's residual).
    """
    dev, B, T, k, D, n_rows = _check_common(rows, alphas, h_A, d_B, r, d_A, row_index)
    act = dtype_code(h_A.dtype, "h_A")
    rdt = dtype_code(rows.dtype, "rows")
    alphas, W_base, b_base = _f32(alphas), _f32(W_base), _f32(b_base)
    gamma = _f32(gamma.reshape(1))
    for name, t in (("alphas", alphas), ("W_base", W_base), ("b_base", b_base), ("gamma", gamma)):
        require_cuda(name, t, dev)
    h_mid = torch.empty((B, T, d_B), dtype=h_A.dtype, device=dev)
    W = torch.empty((B, d_B, d_A), dtype=torch.float32, device=dev) if want_W else None
    if h_A.dtype == torch.float32 and W is not None:
        W_act = W
    else:
        W_act = torch.empty((B, d_B, d_A), dtype=h_A.dtype, device=dev)
    dims = _dims(B, T, k, D, d_A, d_B, r, act, rdt, n_rows)
    lib = _lib.load()
    nbytes = lib.dwa_assemble_workspace_bytes(dims, 0)
    ws = workspace(dev, "assemble_fwd", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_assemble_fwd(stream_of(dev), dims, ptr(rows), ptr(row_index), ptr(alphas),
                                  ptr(h_A), ptr(W_base), ptr(b_base), ptr(gamma), ptr(h_mid),
                                  ptr(W), ptr(W_act), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_assemble_fwd")
    return h_mid, W, W_act


def assemble_apply(rows, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A, *, row_index=None):
    """One ``dwa_assemble_apply`` call: ``h_mid`` only, the Pallas kernel's
    factored form (assembly_pallas.py:85-132) for callers that do not use W
    (generation, train.py:615-616).  Sequences of at most 16 rows never form W;
    longer ones take the ``dwa_assemble_fwd`` path.  Same arguments as
    :func:`assemble_forward`; returns ``h_mid [B,T,d_B]`` in ``h_A``'s dtype.
    """
    dev, B, T, k, D, n_rows = _check_common(rows, alphas, h_A, d_B, r, d_A, row_index)
    act = dtype_code(h_A.dtype, "h_A")
    rdt = dtype_code(rows.dtype, "rows")
    alphas, W_base, b_base = _f32(alphas), _f32(W_base), _f32(b_base)
    gamma = _f32(gamma.reshape(1))
    for name, t in (("alphas", alphas), ("W_base", W_base), ("b_base", b_base), ("gamma", gamma)):
        require_cuda(name, t, dev)
    h_mid = torch.empty((B, T, d_B), dtype=h_A.dtype, device=dev)
    dims = _dims(B, T, k, D, d_A, d_B, r, act, rdt, n_rows)
    lib = _lib.load()
    nbytes = lib.dwa_assemble_apply_workspace_bytes(dims)
    ws = workspace(dev, "assemble_apply", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_assemble_apply(stream_of(dev), dims, ptr(rows), ptr(row_index), ptr(alphas),
                                    ptr(h_A), ptr(W_base), ptr(b_base), ptr(gamma), ptr(h_mid),
                                    ptr(ws), ws.numel())
    _lib.check(rc, "dwa_assemble_apply")
    return h_mid


def assemble_backward(rows, alphas, h_A, W_act, gamma, g_hmid, g_W, d_B, r, d_A, *,
                      row_index=None):
    """One ``dwa_assemble_bwd`` call (the analytic VJP, assembly_pallas.py:246-329).

    Returns ``(g_rows [B,k,D] f32, g_alpha [B,k], g_hA [B,T,d_A], g_W_base,
    g_b_base, g_gamma [1])``.  ``g_W`` may be ``None`` (zero cotangent of W).
    """
    dev, B, T, k, D, n_rows = _check_common(rows, alphas, h_A, d_B, r, d_A, row_index)
    act = dtype_code(h_A.dtype, "h_A")
    rdt = dtype_code(rows.dtype, "rows")
    alphas = _f32(alphas)
    gamma = _f32(gamma.reshape(1))
    if g_hmid.dtype != h_A.dtype:
        g_hmid = g_hmid.to(h_A.dtype)
    g_hmid = g_hmid.contiguous()
    if W_act.dtype != h_A.dtype:
        W_act = W_act.to(h_A.dtype)
    if g_W is not None:
        g_W = _f32(g_W)
    for name, t in (("alphas", alphas), ("W_act", W_act), ("gamma", gamma), ("g_hmid", g_hmid)):
        require_cuda(name, t, dev)
    g_rows = torch.empty((B, k, D), dtype=torch.float32, device=dev)
    g_alpha = torch.empty((B, k), dtype=torch.float32, device=dev)
    g_hA = torch.empty_like(h_A)
    g_W_base = torch.empty((d_B, d_A), dtype=torch.float32, device=dev)
    g_b_base = torch.empty((d_B,), dtype=torch.float32, device=dev)
    g_gamma = torch.empty((1,), dtype=torch.float32, device=dev)
    dims = _dims(B, T, k, D, d_A, d_B, r, act, rdt, n_rows)
    lib = _lib.load()
    nbytes = lib.dwa_assemble_workspace_bytes(dims, 1)
    ws = workspace(dev, "assemble_bwd", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_assemble_bwd(stream_of(dev), dims, ptr(rows), ptr(row_index), ptr(alphas),
                                  ptr(h_A), ptr(W_act), ptr(gamma), ptr(g_hmid), ptr(g_W),
                                  ptr(g_rows), ptr(g_alpha), ptr(g_hA), ptr(g_W_base),
                                  ptr(g_b_base), ptr(g_gamma), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_assemble_bwd")
    return g_rows, g_alpha, g_hA, g_W_base, g_b_base, g_gamma


class _Assemble(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gathered, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A, group):
        h_mid, W, W_act = assemble_forward(gathered, alphas, h_A, W_base, b_base, gamma,
                                           d_B, r, d_A)
        ctx.save_for_backward(gathered, alphas, h_A, W_act, gamma)
        ctx.dims = (d_B, r, d_A)
        ctx.group = group
        ctx.dtypes = (W_base.dtype, b_base.dtype, gamma.dtype, gamma.shape)
        ctx.set_materialize_grads(False)
        return h_mid, W

    @staticmethod
    def backward(ctx, g_hmid, g_W):
        gathered, alphas, h_A, W_act, gamma = ctx.saved_tensors
        d_B, r, d_A = ctx.dims
        if g_hmid is None:
            g_hmid = torch.zeros_like(h_A)
        g_rows, g_alpha, g_hA, g_Wb, g_bb, g_gm = assemble_backward(
            gathered, alphas, h_A, W_act, gamma, g_hmid, g_W, d_B, r, d_A)
        if ctx.group is not False:
            # shard_map transpose of replicated inputs: sum over the data axis
            import torch.distributed as dist
            flat = torch.cat([g_Wb.reshape(-1), g_bb, g_gm])
            dist.all_reduce(flat, group=ctx.group)
            n1, n2 = g_Wb.numel(), g_bb.numel()
            g_Wb = flat[:n1].view_as(g_Wb)
            g_bb = flat[n1:n1 + n2]
            g_gm = flat[n1 + n2:]
        wdt, bdt, gdt, gshape = ctx.dtypes
        return (g_rows.to(gathered.dtype), g_alpha.to(alphas.dtype), g_hA, g_Wb.to(wdt),
                g_bb.to(bdt), g_gm.reshape(gshape).to(gdt), None, None, None, None)


def pallas_assemble(gathered, alphas, h_A, W_base, b_base, gamma, d_B: int, r: int, d_A: int):
    """B200 assembly with a custom VJP; same contract as ``pallas_assemble``
    (src/dwa/assembly_pallas.py:193-222).  Returns ``(h_mid, W)``."""
    return _Assemble.apply(gathered, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A, False)


def shard_pallas_assemble(gathered, alphas, h_A, W_base, b_base, gamma, d_B: int, r: int,
                          d_A: int, mesh=None):
    """Batch-sharded assembly (src/dwa/assembly_pallas.py:339-385).

    One process per GPU: each rank passes its own batch slice of ``gathered``,
    ``alphas`` and ``h_A`` and the replicated ``W_base``, ``b_base``, ``gamma``;
    ``mesh`` is the data-parallel process group (``None``: the default group).
    The forward needs no communication; the backward all-reduces the gradients
    of the replicated parameters, as ``shard_map``'s transpose does.
    """
    return _Assemble.apply(gathered, alphas, h_A, W_base, b_base, gamma, d_B, r, d_A, mesh)


def compute_key_cache(pool_vectors: torch.Tensor, key_proj: torch.Tensor) -> torch.Tensor:
    """``compute_key_cache`` (src/dwa/assembly_pallas.py:392-400, pool.py:37-44):
    keys ``[S, N, d_k]`` f32 = einsum("nd,sda->sna") of the pool ``[N, D]`` and the
    key projections ``[S, D, d_k]`` (both bf16 or both f32), one ``dwa_key_cache``
    GEMM (tcgen05 for bf16)."""
    require_cuda("pool_vectors", pool_vectors)
    dev = pool_vectors.device
    require_cuda("key_proj", key_proj, dev)
    if pool_vectors.dim() != 2 or key_proj.dim() != 3 or key_proj.shape[1] != pool_vectors.shape[1]:
        raise ValueError("pool_vectors must be [N, D] and key_proj [S, D, d_k]")
    if pool_vectors.dtype != key_proj.dtype:
        raise ValueError("pool_vectors and key_proj must have the same dtype")
    N, D = pool_vectors.shape
    S, _, d_k = key_proj.shape
    dims = _lib.KeyCacheDims(N, D, S, d_k, dtype_code(pool_vectors.dtype, "pool_vectors"))
    pool_vectors = pool_vectors.contiguous()
    key_proj = key_proj.contiguous()
    keys = torch.empty((S, N, d_k), dtype=torch.float32, device=dev)
    lib = _lib.load()
    nbytes = lib.dwa_key_cache_workspace_bytes(dims)
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_key_cache_workspace_bytes: {_lib.last_error()}")
    ws = workspace(dev, "key_cache", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_key_cache(stream_of(dev), dims, ptr(pool_vectors), ptr(key_proj), ptr(keys),
                               ptr(ws), ws.numel())
    _lib.check(rc, "dwa_key_cache")
    return keys


def centroid_ema(centroids: torch.Tensor, keys: torch.Tensor, list_offsets: torch.Tensor,
                 decay: float = 0.9) -> torch.Tensor:
    """The centroid update of train.py:318-328 in place: ``centroids [S, C, d_k]
    = decay * centroids + (1 - decay) * mean of each list's keys`` (CSR
    ``list_offsets [C+1]`` into ``keys [S, N, d_k]``).  Returns ``centroids``."""
    require_cuda("centroids", centroids)
    dev = centroids.device
    require_cuda("keys", keys, dev)
    require_cuda("list_offsets", list_offsets, dev)
    S, C, d_k = centroids.shape
    if centroids.dtype != torch.float32 or not centroids.is_contiguous():
        raise ValueError("centroids must be contiguous float32 [S, C, d_k]")
    if keys.dtype != torch.float32 or keys.shape[0] != S or keys.shape[2] != d_k:
        raise ValueError("keys must be float32 [S, N, d_k]")
    if list_offsets.dtype != torch.int64 or list_offsets.numel() != C + 1:
        raise ValueError("list_offsets must be int64 [C+1]")
    keys = keys.contiguous()
    lib = _lib.load()
    ws = workspace(dev, "centroid_ema", 256)
    with torch.cuda.device(dev):
        rc = lib.dwa_centroid_ema(stream_of(dev), S, C, d_k, keys.shape[1], ptr(keys),
                                  ptr(list_offsets.contiguous()), float(decay), ptr(centroids),
                                  ptr(ws), ws.numel())
    _lib.check(rc, "dwa_centroid_ema")
    return centroids
