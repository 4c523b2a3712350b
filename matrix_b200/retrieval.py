"""Multi-aspect IVF retrieval on libdwa's B200 kernels.

Drop-in for ``MultiAspectRetrieval`` (src/dwa/retrieval.py:16-159): the same
parameters (``W_Q [S,d_k,d_A]``, ``aspect_weights [S]``, ``tau``,
``centroids [S,C,d_k]``) and the same call
``(z, pool_keys, lambda_val, is_warmup, mesh=None) -> (alphas, indices, soft_full)``.

Differences, all opt-in or documented:

* ``list_offsets`` (CSR, ``[C+1]`` int64) lets lists have unequal sizes; the
  default is the reference's equal lists ``c*N/C``.
* ``want_soft_full=False`` skips the full-pool soft scores, which the reference
  computes on every call and XLA drops when no loss reads them.
* Ties between bit-identical scores go to the lower pool row (the reference's
  ``lax.top_k`` prefers the lower candidate position); with distinct scores the
  two rules select the same rows in the same order.
* ``retrieve`` itself carries no gradient; ``retrieve_with_grad`` is the
  differentiable op, whose backward is ``dwa_retrieve_bwd``
  (``retrieve_backward``).  ``MultiAspectRetrieval`` takes it whenever grad
  mode is on and one of its inputs or parameters requires grad.
"""

from __future__ import annotations

import torch

from . import _lib
from .config import DWAConfig
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace


def equal_list_offsets(N: int, C: int, device) -> torch.Tensor:
    if N % C:
        raise ValueError(f"N={N} must be divisible by C={C} for equal lists")
    return (torch.arange(C + 1, dtype=torch.int64, device=device) * (N // C)).contiguous()


def sequence_mean(h_A: torch.Tensor) -> torch.Tensor:
    """The retrieval query input ``z = h_A.mean(axis=1)`` (model.py:171):
    ``h_A [B, T, d_A]`` f32 or bf16 -> ``z [B, d_A]`` f32, summed in fp32 in a
    fixed order (``dwa_sequence_mean``)."""
    require_cuda("h_A", h_A)
    if h_A.dim() != 3:
        raise ValueError("h_A must be [B, T, d_A]")
    h_A = h_A.contiguous()
    B, T, d = h_A.shape
    z = torch.empty((B, d), dtype=torch.float32, device=h_A.device)
    with torch.cuda.device(h_A.device):
        rc = _lib.load().dwa_sequence_mean(stream_of(h_A.device), B, T, d, dtype_code(h_A.dtype, "h_A"),
                                           ptr(h_A), ptr(z))
    _lib.check(rc, "dwa_sequence_mean")
    return z


def _call_args(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, *, k, m, T, use_ivf,
               list_offsets, max_list):
    """Checked arguments of one retrieval call (forward or VJP): the dims
    struct and the float32 / int64 device tensors the C ABI takes."""
    require_cuda("z", z)
    dev = z.device
    require_cuda("pool_keys", pool_keys, dev)
    if pool_keys.dtype != torch.float32 or pool_keys.dim() != 3:
        raise ValueError("pool_keys must be float32 [S, N, d_k]")
    S, N, d_k = pool_keys.shape
    B, d_A = z.shape
    if tuple(W_Q.shape) != (S, d_k, d_A):
        raise ValueError(f"W_Q must be [S={S}, d_k={d_k}, d_A={d_A}], got {tuple(W_Q.shape)}")
    if k > N:
        raise ValueError(f"k={k} > N={N}")
    C = centroids.shape[1] if (use_ivf and centroids is not None) else 1
    if use_ivf:
        require_cuda("centroids", centroids, dev)
        if tuple(centroids.shape) != (S, C, d_k) or centroids.dtype != torch.float32:
            raise ValueError("centroids must be float32 [S, C, d_k]")
        if list_offsets is None:
            list_offsets = equal_list_offsets(N, C, dev)
            max_list = N // C
            if min(m, C) * (N // C) < k:
                raise ValueError("fewer IVF candidates than k")
        require_cuda("list_offsets", list_offsets, dev)
        if list_offsets.dtype != torch.int64 or list_offsets.numel() != C + 1:
            raise ValueError("list_offsets must be int64 [C+1]")
        if max_list is None:
            max_list = int((list_offsets[1:] - list_offsets[:-1]).max().item())
    lam = lambda_val if isinstance(lambda_val, torch.Tensor) else torch.tensor(
        [float(lambda_val)], dtype=torch.float32, device=dev)
    return dict(
        dims=_lib.RetrieveDims(B, S, d_k, d_A, C, m, k, int(max_list or 0), N, float(T),
                               dtype_code(z.dtype, "z")),
        lam=lam.reshape(1).float().contiguous(), tau=tau.reshape(1).float().contiguous(),
        W_Q=W_Q.float().contiguous(), aw=aspect_weights.float().contiguous(),
        list_offsets=list_offsets, dev=dev, B=B, N=N, S=S, d_k=d_k, d_A=d_A)


def retrieve(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, is_warmup, *, k, m, T,
             use_ivf=True, list_offsets=None, max_list=None, want_soft_full=True):
    """One ``dwa_retrieve`` call.  Returns ``(alphas [B,k] f32, indices [B,k]
    int32, soft_full [B,N] f32 or None)``."""
    a = _call_args(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, k=k, m=m, T=T,
                   use_ivf=use_ivf, list_offsets=list_offsets, max_list=max_list)
    dev, B, N = a["dev"], a["B"], a["N"]
    alphas = torch.empty((B, k), dtype=torch.float32, device=dev)
    indices = torch.empty((B, k), dtype=torch.int32, device=dev)
    soft_full = torch.empty((B, N), dtype=torch.float32, device=dev) if want_soft_full else None
    lib = _lib.load()
    nbytes = lib.dwa_retrieve_workspace_bytes(a["dims"], int(use_ivf), int(want_soft_full))
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_retrieve_workspace_bytes: {_lib.last_error()}")
    ws = workspace(dev, "retrieve", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve(stream_of(dev), a["dims"], int(use_ivf), int(bool(is_warmup)), ptr(a["lam"]),
                              ptr(z), ptr(a["W_Q"]), ptr(a["aw"]), ptr(a["tau"]),
                              ptr(centroids) if use_ivf else None,
                              ptr(a["list_offsets"]) if use_ivf else None, ptr(pool_keys),
                              ptr(alphas), ptr(indices), ptr(soft_full), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve")
    return alphas, indices, soft_full


def retrieve_backward(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, is_warmup,
                      alphas, indices, soft_full, g_alphas, g_soft_full, *, k, m, T, use_ivf=True,
                      list_offsets=None, max_list=None, want_key_grad=False):
    """One ``dwa_retrieve_bwd`` call: the VJP of ``retrieve`` (retrieval.py:64-158)
    for the cotangents ``g_alphas [B,k]`` and ``g_soft_full [B,N]`` (either may
    be ``None``), given the forward's ``alphas``, ``indices`` and normalised
    ``soft_full``.  Returns ``dict(g_z [B,d_A], g_W_Q [S,d_k,d_A],
    g_aspect_weights [S], g_tau [], g_pool_keys [S,N,d_k] or None)``, float32."""
    a = _call_args(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, k=k, m=m, T=T,
                   use_ivf=use_ivf, list_offsets=list_offsets, max_list=max_list)
    dev = a["dev"]
    f32 = dict(dtype=torch.float32, device=dev)

    def opt(t, shape, name):
        if t is None:
            return None
        require_cuda(name, t, dev)
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must be {shape}, got {tuple(t.shape)}")
        return t.float().contiguous()

    g_alphas = opt(g_alphas, (a["B"], k), "g_alphas")
    g_soft_full = opt(g_soft_full, (a["B"], a["N"]), "g_soft_full")
    if g_soft_full is not None and soft_full is None:
        raise ValueError("g_soft_full needs the forward's soft_full")
    out = dict(g_z=torch.empty((a["B"], a["d_A"]), **f32), g_W_Q=torch.empty(tuple(W_Q.shape), **f32),
               g_aspect_weights=torch.empty((a["S"],), **f32), g_tau=torch.empty((), **f32),
               g_pool_keys=torch.empty(tuple(pool_keys.shape), **f32) if want_key_grad else None)
    lib = _lib.load()
    nbytes = lib.dwa_retrieve_bwd_workspace_bytes(a["dims"], int(use_ivf))
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_retrieve_bwd_workspace_bytes: {_lib.last_error()}")
    ws = workspace(dev, "retrieve_bwd", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve_bwd(
            stream_of(dev), a["dims"], int(use_ivf), int(bool(is_warmup)), ptr(a["lam"]), ptr(z), ptr(a["W_Q"]),
            ptr(a["aw"]), ptr(a["tau"]), ptr(centroids) if use_ivf else None,
            ptr(a["list_offsets"]) if use_ivf else None, ptr(pool_keys),
            ptr(alphas.float().contiguous()) if alphas is not None else None,
            ptr(indices.int().contiguous()) if indices is not None else None,
            ptr(soft_full.float().contiguous()) if soft_full is not None else None,
            ptr(g_alphas), ptr(g_soft_full), ptr(out["g_z"]), ptr(out["g_W_Q"]), ptr(out["g_aspect_weights"]),
            ptr(out["g_tau"]), ptr(out["g_pool_keys"]), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve_bwd")
    return out


class _RetrieveFunction(torch.autograd.Function):
    """``retrieve`` with its VJP: gradients reach z, W_Q, aspect_weights, tau
    and (when it requires grad) the key cache, as ``jax.grad`` of the
    reference's retrieval gives them."""

    @staticmethod
    def forward(ctx, z, W_Q, aspect_weights, tau, pool_keys, centroids, list_offsets, lambda_val, opts):
        alphas, indices, soft_full = retrieve(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val,
                                              opts["is_warmup"], k=opts["k"], m=opts["m"], T=opts["T"],
                                              use_ivf=opts["use_ivf"], list_offsets=list_offsets,
                                              max_list=opts["max_list"], want_soft_full=opts["want_soft_full"])
        ctx.save_for_backward(z, W_Q, aspect_weights, tau, pool_keys, alphas, indices,
                              soft_full if soft_full is not None else torch.empty(0, device=z.device))
        ctx.centroids, ctx.list_offsets, ctx.lambda_val, ctx.opts = centroids, list_offsets, lambda_val, opts
        ctx.has_sf = soft_full is not None
        ctx.mark_non_differentiable(indices)
        return alphas, indices, soft_full

    @staticmethod
    def backward(ctx, g_alphas, g_indices, g_soft_full):
        z, W_Q, aw, tau, pool_keys, alphas, indices, soft_full = ctx.saved_tensors
        o = ctx.opts
        g = retrieve_backward(z, W_Q, aw, tau, ctx.centroids, pool_keys, ctx.lambda_val, o["is_warmup"], alphas,
                              indices, soft_full if ctx.has_sf else None, g_alphas,
                              g_soft_full if ctx.has_sf else None, k=o["k"], m=o["m"], T=o["T"],
                              use_ivf=o["use_ivf"], list_offsets=ctx.list_offsets, max_list=o["max_list"],
                              want_key_grad=ctx.needs_input_grad[4])
        return (g["g_z"].to(z.dtype), g["g_W_Q"], g["g_aspect_weights"], g["g_tau"].reshape(tau.shape),
                g["g_pool_keys"], None, None, None, None)


def retrieve_with_grad(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, is_warmup, *, k, m, T,
                       use_ivf=True, list_offsets=None, max_list=None, want_soft_full=True):
    """``retrieve`` as a differentiable op (``torch.autograd``): ``alphas`` and
    ``soft_full`` carry gradients back through ``dwa_retrieve_bwd``."""
    opts = dict(is_warmup=bool(is_warmup), k=k, m=m, T=T, use_ivf=use_ivf, max_list=max_list,
                want_soft_full=want_soft_full)
    return _RetrieveFunction.apply(z, W_Q, aspect_weights, tau, pool_keys, centroids, list_offsets, lambda_val,
                                   opts)


class MultiAspectRetrieval:
    """B200 counterpart of ``MultiAspectRetrieval`` (src/dwa/retrieval.py:16-159)."""

    def __init__(self, cfg: DWAConfig, device=None, generator: torch.Generator | None = None):
        self.cfg = cfg
        dev = torch.device(device if device is not None else "cuda")
        g = generator
        # retrieval.py:35-46 initialisation scales
        self.W_Q = (torch.randn(cfg.S, cfg.d_k, cfg.d_A, generator=g) * cfg.d_A ** -0.5).to(dev)
        self.aspect_weights = torch.zeros(cfg.S, device=dev)
        self.tau = torch.zeros((), device=dev)
        self.centroids = (torch.randn(cfg.S, cfg.C, cfg.d_k, generator=g) * cfg.d_k ** -0.5).to(dev)
        self.list_offsets = None
        self.max_list = None

    def set_lists(self, list_offsets: torch.Tensor, max_list: int | None = None) -> None:
        """Use CSR lists ``[C+1]`` instead of the equal lists of the reference."""
        self.list_offsets = list_offsets
        self.max_list = max_list

    def __call__(self, z, pool_keys, lambda_val, is_warmup: bool, mesh=None, *,
                 want_soft_full: bool = True):
        """``mesh``: ``None`` (one device) or a ``matrix_b200.sharded.RowShard``,
        in which case ``pool_keys`` holds this rank's rows and soft_full is its
        slice (the reference's ``mesh`` branch, retrieval.py:74-79)."""
        cfg = self.cfg
        if mesh is not None:
            from .sharded import RowShard, sharded_retrieve
            if not isinstance(mesh, RowShard):
                raise TypeError("mesh must be a matrix_b200.sharded.RowShard")
            offs = self.list_offsets
            if cfg.use_ivf and offs is None:
                offs = equal_list_offsets(mesh.n_global, cfg.C, z.device)
            return sharded_retrieve(z, self.W_Q, self.aspect_weights, self.tau, self.centroids,
                                    pool_keys, offs, lambda_val, is_warmup, mesh, k=cfg.k_max,
                                    m=cfg.m, T=cfg.T, max_list=self.max_list, use_ivf=cfg.use_ivf,
                                    want_soft_full=want_soft_full)
        diff = torch.is_grad_enabled() and any(
            t.requires_grad for t in (z, self.W_Q, self.aspect_weights, self.tau, pool_keys))
        return (retrieve_with_grad if diff else retrieve)(
            z, self.W_Q, self.aspect_weights, self.tau, self.centroids, pool_keys, lambda_val, is_warmup,
            k=cfg.k_max, m=cfg.m, T=cfg.T, use_ivf=cfg.use_ivf, list_offsets=self.list_offsets,
            max_list=self.max_list, want_soft_full=want_soft_full)
