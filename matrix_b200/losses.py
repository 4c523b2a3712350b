"""Auxiliary losses of DWA training on libdwa's B200 kernels.

Drop-in for ``aux_losses`` (src/dwa/losses.py:9-73): the same inputs
(``alphas``, ``indices``, ``pool_keys``, ``W``, ``W_base``, ``soft_full``) and
the same five outputs (``l_util``, ``l_div``, ``l_norm``, ``l_sparse``,
``total_aux``), with the weights of ``TrainConfig`` (config.py:181-184) as
keyword arguments.  ``aux_losses_with_grad`` returns ``total_aux`` as a
differentiable tensor whose backward is the library's gradient pass.
"""

from __future__ import annotations

import torch

from . import _lib
from .runtime import ptr, require_cuda, stream_of, workspace

DEFAULT_LAMBDAS = dict(lambda_util=0.01, lambda_div=0.01, lambda_norm=0.001, lambda_sparse=0.001)
NAMES = ("l_util", "l_div", "l_norm", "l_sparse", "total_aux")


def _call(alphas, indices, pool_keys, W, W_base, soft_full, lambdas, *, grads, key_grad_into=None):
    require_cuda("alphas", alphas)
    dev = alphas.device
    for name, t in (("indices", indices), ("pool_keys", pool_keys), ("W", W), ("W_base", W_base),
                    ("soft_full", soft_full)):
        require_cuda(name, t, dev)
    B, k = alphas.shape
    S, N, d_k = pool_keys.shape
    _, d_B, d_A = W.shape
    if tuple(indices.shape) != (B, k) or tuple(soft_full.shape) != (B, N) or tuple(W_base.shape) != (d_B, d_A):
        raise ValueError("aux_losses: inconsistent shapes")
    alphas = alphas.float().contiguous()
    indices = indices.int().contiguous()
    pool_keys = pool_keys.float().contiguous()
    W = W.float().contiguous()
    W_base = W_base.float().contiguous()
    soft_full = soft_full.float().contiguous()
    dims = _lib.AuxDims(B, k, S, d_k, d_B, d_A, N)
    lam = _lib.AuxWeights(lambdas["lambda_util"], lambdas["lambda_div"], lambdas["lambda_norm"],
                          lambdas["lambda_sparse"])
    losses = torch.empty(5, dtype=torch.float32, device=dev)
    g = {}
    if grads:
        g = dict(g_alphas=torch.empty_like(alphas), g_soft_full=torch.empty_like(soft_full),
                 g_W=torch.empty_like(W), g_W_base=torch.empty_like(W_base))
    if key_grad_into is not None:
        require_cuda("key_grad_into", key_grad_into, dev)
        if key_grad_into.dtype != torch.float32 or tuple(key_grad_into.shape) != (S, N, d_k) \
                or not key_grad_into.is_contiguous():
            raise ValueError("key_grad_into must be a contiguous float32 [S, N, d_k] tensor")
    lib = _lib.load()
    nbytes = lib.dwa_aux_losses_workspace_bytes(dims)
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_aux_losses_workspace_bytes: {_lib.last_error()}")
    ws = workspace(dev, "aux_losses", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_aux_losses(stream_of(dev), dims, lam, ptr(alphas), ptr(indices), ptr(pool_keys), ptr(W),
                                ptr(W_base), ptr(soft_full), ptr(losses), ptr(g.get("g_alphas")),
                                ptr(g.get("g_soft_full")), ptr(g.get("g_W")), ptr(g.get("g_W_base")),
                                ptr(key_grad_into), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_aux_losses")
    return dict(zip(NAMES, losses.unbind())), g


def aux_losses(alphas, indices, pool_keys, W, W_base, soft_full, **lambdas):
    """The five losses of ``aux_losses`` (losses.py:9-73) as 0-d float32 tensors."""
    lam = {**DEFAULT_LAMBDAS, **lambdas}
    return _call(alphas, indices, pool_keys, W, W_base, soft_full, lam, grads=False)[0]


def aux_losses_and_grads(alphas, indices, pool_keys, W, W_base, soft_full, *, key_grad_into=None, **lambdas):
    """Losses and the gradients of ``total_aux`` w.r.t. alphas, soft_full, W and
    W_base; with ``key_grad_into`` ([S,N,d_k] f32) the gradient w.r.t. the key
    cache is added into it."""
    lam = {**DEFAULT_LAMBDAS, **lambdas}
    return _call(alphas, indices, pool_keys, W, W_base, soft_full, lam, grads=True, key_grad_into=key_grad_into)


class _AuxLossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, alphas, soft_full, W, W_base, pool_keys, indices, lam):
        losses, g = _call(alphas, indices, pool_keys, W, W_base, soft_full, lam, grads=True)
        ctx.save_for_backward(g["g_alphas"], g["g_soft_full"], g["g_W"], g["g_W_base"])
        ctx.key_args = (alphas, indices, pool_keys, W, W_base, soft_full, lam)
        ctx.want_keys = pool_keys.requires_grad
        return losses["total_aux"], torch.stack([losses[n] for n in NAMES[:4]])

    @staticmethod
    def backward(ctx, g_total, g_parts):
        ga, gs, gw, gwb = ctx.saved_tensors
        gk = None
        if ctx.want_keys:
            alphas, indices, pool_keys, W, W_base, soft_full, lam = ctx.key_args
            gk = torch.zeros(tuple(pool_keys.shape), dtype=torch.float32, device=pool_keys.device)
            _call(alphas, indices, pool_keys, W, W_base, soft_full, lam, grads=False, key_grad_into=gk)
            gk = gk * g_total
        return ga * g_total, gs * g_total, gw * g_total, gwb * g_total, gk, None, None


def aux_losses_with_grad(alphas, indices, pool_keys, W, W_base, soft_full, **lambdas):
    """``total_aux`` as a differentiable 0-d tensor and the four losses (no
    gradient) as a dict."""
    lam = {**DEFAULT_LAMBDAS, **lambdas}
    total, parts = _AuxLossFunction.apply(alphas, soft_full, W, W_base, pool_keys, indices, lam)
    return total, dict(zip(NAMES[:4], parts.detach().unbind()))


def sharded_aux_losses_and_grads(alphas, indices, local_keys, W_local, W_base, soft_local, *, row_lo, n_global,
                                 group=None, key_grad_into=None, reduce=None, **lambdas):
    """``aux_losses`` and its gradients over a row-sharded pool: this rank holds
    the key / soft_full rows ``[row_lo, row_lo + rows)`` and the assembled W of
    its own sequences.  One all-reduce (``reduce``; default ``dist.all_reduce``
    over ``group``) sums the ranks' ``l_util`` / ``l_norm`` shares, the winners'
    aspect-mean keys and ``g_W_base``.  Returns ``(losses, grads)``: the losses
    and ``g_alphas`` / ``g_W_base`` are the same on every rank; ``g_soft_full``
    and ``g_W`` are this rank's slices; the key gradient of its rows is added
    into ``key_grad_into``."""
    import torch.distributed as dist
    lam = {**DEFAULT_LAMBDAS, **lambdas}
    dev = alphas.device
    B, k = alphas.shape
    S, n_loc, d_k = local_keys.shape
    d_B, d_A = W_base.shape
    w_batch = 0 if W_local is None else W_local.shape[0]
    dims = _lib.AuxDims(B, k, S, d_k, d_B, d_A, max(n_loc, 1))
    shard = _lib.AuxShard(int(row_lo), int(n_global), int(w_batch))
    weights = _lib.AuxWeights(lam["lambda_util"], lam["lambda_div"], lam["lambda_norm"], lam["lambda_sparse"])
    idx = indices.int().contiguous()
    f32 = dict(dtype=torch.float32, device=dev)
    part, rk = torch.zeros(2, **f32), torch.zeros((B, k, d_k), **f32)
    g = dict(g_alphas=torch.empty((B, k), **f32), g_soft_full=torch.zeros((B, n_loc), **f32),
             g_W=torch.empty((w_batch, d_B, d_A), **f32), g_W_base=torch.zeros((d_B, d_A), **f32))
    lib = _lib.load()
    ws = workspace(dev, "aux_losses_sharded", lib.dwa_aux_losses_workspace_bytes(dims))
    if n_loc > 0 or w_batch > 0:
        keys = local_keys if n_loc > 0 else torch.zeros((S, 1, d_k), **f32)
        soft = soft_local.float().contiguous() if n_loc > 0 else torch.zeros((B, 1), **f32)
        with torch.cuda.device(dev):
            rc = lib.dwa_aux_losses_local(stream_of(dev), dims, shard, weights, ptr(idx), ptr(keys.contiguous()),
                                          ptr(W_local.float().contiguous()) if w_batch else None,
                                          ptr(W_base.float().contiguous()), ptr(soft), ptr(part), ptr(rk),
                                          ptr(g["g_soft_full"]) if n_loc > 0 else None,
                                          ptr(g["g_W"]) if w_batch else None, ptr(g["g_W_base"]), ptr(ws),
                                          ws.numel())
        _lib.check(rc, "dwa_aux_losses_local")
    if reduce is None:
        world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if world > 1:
            for t in (part, rk, g["g_W_base"]):
                dist.all_reduce(t, group=group)
    else:
        part, rk, g["g_W_base"] = reduce(part, rk, g["g_W_base"])
    losses = torch.empty(5, **f32)
    with torch.cuda.device(dev):
        rc = lib.dwa_aux_losses_finish(stream_of(dev), dims, shard, weights, ptr(alphas.float().contiguous()), ptr(idx),
                                       ptr(part.contiguous()), ptr(rk.contiguous()), ptr(losses), ptr(g["g_alphas"]),
                                       ptr(key_grad_into) if (key_grad_into is not None and n_loc > 0) else None,
                                       ptr(ws), ws.numel())
    _lib.check(rc, "dwa_aux_losses_finish")
    return dict(zip(NAMES, losses.unbind())), g
