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
* The outputs carry no gradient: the retrieval VJP is not part of this path.
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


def retrieve(z, W_Q, aspect_weights, tau, centroids, pool_keys, lambda_val, is_warmup, *, k, m, T,
             use_ivf=True, list_offsets=None, max_list=None, want_soft_full=True):
    """One ``dwa_retrieve`` call.  Returns ``(alphas [B,k] f32, indices [B,k]
    int32, soft_full [B,N] f32 or None)``."""
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
    lam = lam.reshape(1).float().contiguous()
    tau_t = tau.reshape(1).float().contiguous()
    W_Q = W_Q.float().contiguous()
    aw = aspect_weights.float().contiguous()
    zdt = dtype_code(z.dtype, "z")
    dims = _lib.RetrieveDims(B, S, d_k, d_A, C, m, k, int(max_list or 0), N, float(T), zdt)
    alphas = torch.empty((B, k), dtype=torch.float32, device=dev)
    indices = torch.empty((B, k), dtype=torch.int32, device=dev)
    soft_full = torch.empty((B, N), dtype=torch.float32, device=dev) if want_soft_full else None
    lib = _lib.load()
    nbytes = lib.dwa_retrieve_workspace_bytes(dims, int(use_ivf), int(want_soft_full))
    if nbytes == 0:
        raise _lib.DwaError(f"dwa_retrieve_workspace_bytes: {_lib.last_error()}")
    ws = workspace(dev, "retrieve", nbytes)
    with torch.cuda.device(dev):
        rc = lib.dwa_retrieve(stream_of(dev), dims, int(use_ivf), int(bool(is_warmup)), ptr(lam),
                              ptr(z), ptr(W_Q), ptr(aw), ptr(tau_t),
                              ptr(centroids) if use_ivf else None,
                              ptr(list_offsets) if use_ivf else None, ptr(pool_keys),
                              ptr(alphas), ptr(indices), ptr(soft_full), ptr(ws), ws.numel())
    _lib.check(rc, "dwa_retrieve")
    return alphas, indices, soft_full


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
        return retrieve(z, self.W_Q, self.aspect_weights, self.tau, self.centroids, pool_keys,
                        lambda_val, is_warmup, k=cfg.k_max, m=cfg.m, T=cfg.T, use_ivf=cfg.use_ivf,
                        list_offsets=self.list_offsets, max_list=self.max_list,
                        want_soft_full=want_soft_full)
