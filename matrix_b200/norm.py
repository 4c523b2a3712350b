"""RMSNorm after the assembly on libdwa's kernels.

The reference normalises the assembly output with flax's ``nnx.RMSNorm(d_B)``
(the assembler's ``layer_norm``, src/dwa/assembly.py:29, applied at
src/dwa/model.py:207-219): ``y = x * (rsqrt(mean(x^2) + eps) * scale)`` with
``eps = 1e-6`` and a learned ``scale [d]`` initialised to ones.  ``rms_norm`` is
that op with its VJP (``dwa_rmsnorm_fwd`` / ``dwa_rmsnorm_bwd``); ``RMSNorm``
holds the scale like the flax module.
"""

from __future__ import annotations

import torch

from . import _lib
from .runtime import dtype_code, ptr, require_cuda, stream_of, workspace


def rms_norm_forward(x: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6, out_dtype=None):
    """``(y, rstd)``: ``y`` like ``x`` in ``out_dtype`` (default: flax's promotion
    of ``x`` with the fp32 scale, i.e. float32), ``rstd [rows]`` f32."""
    require_cuda("x", x)
    dev = x.device
    require_cuda("scale", scale, dev)
    d = x.shape[-1]
    if scale.shape != (d,) or scale.dtype != torch.float32:
        raise ValueError("scale must be float32 [d]")
    out_dtype = torch.float32 if out_dtype is None else out_dtype
    xc = x.contiguous()
    rows = xc.numel() // d
    y = torch.empty(x.shape, dtype=out_dtype, device=dev)
    rstd = torch.empty(rows, dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.dwa_rmsnorm_fwd(stream_of(dev), rows, d, dtype_code(x.dtype, "x"), dtype_code(out_dtype, "y"),
                                 ptr(xc), ptr(scale.contiguous()), float(eps), ptr(y), ptr(rstd))
    _lib.check(rc, "dwa_rmsnorm_fwd")
    return y, rstd


def rms_norm_backward(x: torch.Tensor, scale: torch.Tensor, rstd: torch.Tensor, g_y: torch.Tensor):
    """``(g_x, g_scale)`` for ``g_y = dL/dy``."""
    require_cuda("x", x)
    dev = x.device
    d = x.shape[-1]
    xc, gc = x.contiguous(), g_y.contiguous()
    rows = xc.numel() // d
    g_x = torch.empty(x.shape, dtype=x.dtype, device=dev)
    g_scale = torch.empty(d, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = workspace(dev, "rmsnorm_bwd", lib.dwa_rmsnorm_bwd_workspace_bytes(rows, d))
    with torch.cuda.device(dev):
        rc = lib.dwa_rmsnorm_bwd(stream_of(dev), rows, d, dtype_code(x.dtype, "x"), dtype_code(gc.dtype, "g_y"),
                                 ptr(xc), ptr(scale.contiguous()), ptr(rstd), ptr(gc), ptr(g_x), ptr(g_scale),
                                 ptr(ws), ws.numel())
    _lib.check(rc, "dwa_rmsnorm_bwd")
    return g_x, g_scale


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, eps, out_dtype):
        y, rstd = rms_norm_forward(x, scale, eps, out_dtype)
        ctx.save_for_backward(x, scale, rstd)
        return y

    @staticmethod
    def backward(ctx, g_y):
        x, scale, rstd = ctx.saved_tensors
        g_x, g_scale = rms_norm_backward(x, scale, rstd, g_y)
        return g_x, g_scale, None, None


def rms_norm(x: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6, out_dtype=None) -> torch.Tensor:
    """Differentiable RMSNorm over the last axis (flax ``nnx.RMSNorm`` semantics)."""
    return _RMSNorm.apply(x, scale, float(eps), out_dtype)


class RMSNorm(torch.nn.Module):
    """``nnx.RMSNorm(num_features, epsilon=1e-6)`` counterpart: a ``scale [d]``
    parameter initialised to ones."""

    def __init__(self, num_features: int, epsilon: float = 1e-6, device=None):
        super().__init__()
        self.epsilon = epsilon
        self.scale = torch.nn.Parameter(torch.ones(num_features, dtype=torch.float32, device=device))

    def forward(self, x: torch.Tensor, out_dtype=None) -> torch.Tensor:
        return rms_norm(x, self.scale, self.epsilon, out_dtype)
