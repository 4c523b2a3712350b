"""A NumPy stand-in for the small part of ``jax`` / ``flax.nnx`` that the
reference's hot-path files use, so that those files can be executed unchanged in
a container without JAX.

Used only by ``make_golden.py`` to produce golden vectors from the reference's
own source (``src/dwa/retrieval.py``, ``src/dwa/assembly_pallas.py``,
``src/dwa/config.py``).  Only the primitives those files call are provided, each
with the documented semantics of its JAX counterpart:

* ``jax.numpy``: NumPy itself (einsum, matmul, linalg.norm, take_along_axis, ...)
* ``jax.nn.softmax``: ``exp(x - max) / sum``; ``jax.nn.sigmoid``: ``1/(1+exp(-x))``
* ``jax.lax.top_k``: descending values, ties to the lower position
* ``jax.lax.cond``: eager branch selection; ``jax.vmap``: loop + stack
* ``jax.custom_vjp``: calls the primal; ``defvjp`` records the rules
* ``jax.experimental.pallas.pallas_call``: runs the kernel body once per grid
  index on NumPy block views selected by each ``BlockSpec`` (the semantics of
  Pallas interpret mode).  Output blocks no grid step writes stay NaN, which
  exposes the reference's ``B % 8`` tail gap.
* ``flax.nnx.Module`` / ``Variable`` / ``Param``: plain attribute holders.

What this does not cover: XLA's own rounding (fused reductions, bf16 rules).
"""

from __future__ import annotations

import sys
import types

import numpy as np


class _Ref:
    """A Pallas ref over a NumPy block: ``ref[...]`` reads, ``ref[...] = x`` writes."""

    def __init__(self, arr):
        self.arr = arr

    def __getitem__(self, idx):
        return self.arr[idx]

    def __setitem__(self, idx, val):
        self.arr[idx] = val


class BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)


def _block_slices(spec: BlockSpec, grid_idx):
    blk = spec.index_map(*grid_idx)
    if not isinstance(blk, tuple):
        blk = (blk,)
    return tuple(slice(int(i) * bs, (int(i) + 1) * bs) for i, bs in zip(blk, spec.block_shape))


def pallas_call(kernel, out_shape, in_specs, out_specs, grid, **_):
    grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)

    def run(*args):
        out = np.full(out_shape.shape, np.nan, dtype=out_shape.dtype)
        for gi in np.ndindex(*grid):
            ins = [_Ref(np.asarray(a)[_block_slices(s, gi)].copy()) for a, s in zip(args, in_specs)]
            o_sl = _block_slices(out_specs, gi)
            o_ref = _Ref(out[o_sl].copy())
            kernel(*ins, o_ref)
            out[o_sl] = o_ref.arr
        return out

    return run


def _top_k(x, k):
    order = np.argsort(-x, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(x, order, axis=-1), order


def _softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _cond(pred, true_fun, false_fun, *operands):
    return true_fun(*operands) if bool(pred) else false_fun(*operands)


def _vmap(fun):
    def mapped(x):
        return np.stack([fun(x[i]) for i in range(x.shape[0])])
    return mapped


class custom_vjp:
    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.nondiff_argnums = tuple(nondiff_argnums)
        self.fwd = self.bwd = None

    def __call__(self, *args):
        return self.fun(*args)

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd


class _Module:
    pass


class _Variable:
    def __init__(self, value):
        self.value = np.asarray(value)

    def __getitem__(self, idx):
        return self.value[idx]

    def __setitem__(self, idx, v):
        self.value[idx] = v


def install():
    """Register the stand-in modules in ``sys.modules`` (idempotent)."""
    if "jax" in sys.modules and getattr(sys.modules["jax"], "_numpy_stand_in", False):
        return
    import ml_dtypes

    jnp = types.ModuleType("jax.numpy")
    for name in dir(np):
        if not name.startswith("_"):
            setattr(jnp, name, getattr(np, name))
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.ndarray = np.ndarray

    nn = types.ModuleType("jax.nn")
    nn.softmax, nn.sigmoid = _softmax, _sigmoid
    lax = types.ModuleType("jax.lax")
    lax.top_k, lax.cond = _top_k, _cond
    random = types.ModuleType("jax.random")
    experimental = types.ModuleType("jax.experimental")
    pallas = types.ModuleType("jax.experimental.pallas")
    pallas.pallas_call, pallas.BlockSpec = pallas_call, BlockSpec
    experimental.pallas = pallas

    jax = types.ModuleType("jax")
    jax._numpy_stand_in = True
    jax.numpy, jax.nn, jax.lax, jax.random, jax.experimental = jnp, nn, lax, random, experimental
    jax.vmap, jax.custom_vjp, jax.ShapeDtypeStruct = _vmap, custom_vjp, ShapeDtypeStruct

    nnx = types.ModuleType("flax.nnx")
    nnx.Module, nnx.Variable, nnx.Param = _Module, _Variable, _Variable
    nnx.Rngs = type("Rngs", (), {})
    flax = types.ModuleType("flax")
    flax.nnx = nnx

    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.nn": nn, "jax.lax": lax, "jax.random": random,
        "jax.experimental": experimental, "jax.experimental.pallas": pallas,
        "flax": flax, "flax.nnx": nnx,
    })


def load_reference_modules(src_dwa_dir: str):
    """Import ``config``, ``retrieval`` and ``assembly_pallas`` from the reference's
    ``src/dwa`` directory as the package ``dwa_reference`` without running its
    ``__init__`` (which imports the transformer halves and the trainer).
    """
    import importlib

    install()
    pkg = types.ModuleType("dwa_reference")
    pkg.__path__ = [src_dwa_dir]
    sys.modules["dwa_reference"] = pkg
    return (importlib.import_module("dwa_reference.config"),
            importlib.import_module("dwa_reference.retrieval"),
            importlib.import_module("dwa_reference.assembly_pallas"))
