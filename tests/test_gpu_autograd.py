"""The Python custom-VJP entry points, called the way the reference's model
calls them (src/dwa/model.py:202-219): ``pallas_assemble`` (the jax.custom_vjp
of src/dwa/assembly_pallas.py:193-222, 332) and ``shard_pallas_assemble``
(the batch-sharded shard_map of :339-385), differentiated by torch.autograd.

The loss is ``<h_mid, g_hmid> + <W, g_W>``, so autograd hands the backward
exactly the cotangents the oracle's VJP receives; all six input gradients
must match the float64 oracle (rtol 1e-5 in float32, 2e-2 in bfloat16).
``shard_pallas_assemble`` runs on a one-rank NCCL process group: its backward
all-reduces the replicated parameters' gradients over the group and must
equal ``pallas_assemble``'s.
"""

from __future__ import annotations

import socket

import numpy as np
import pytest

from conftest import assert_close
from test_gpu_assembly import BF16_TOL, CASES, F32_TOL, _dev, _np, _oracle, _setup

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _leaves(cfg, x, idx, alphas):
    act = torch.bfloat16 if cfg.compute_dtype == "bfloat16" else torch.float32
    pool_dt = torch.bfloat16 if cfg.bf16_pool else torch.float32
    gathered = _dev(x.pool, pool_dt)[_dev(idx).long()].contiguous()
    leaves = [gathered, _dev(alphas), _dev(x.h_A, act), _dev(x.W_base), _dev(x.b_base),
              torch.tensor(x.gamma, dtype=torch.float32).cuda()]
    return [t.detach().requires_grad_(True) for t in leaves], act


def _grads(fn, cfg, x, idx, alphas):
    leaves, act = _leaves(cfg, x, idx, alphas)
    h_mid, W = fn(*leaves, cfg.d_B, cfg.r, cfg.d_A)
    loss = (h_mid.float() * _dev(x.g_hmid, act).float()).sum() + (W * _dev(x.g_W)).sum()
    loss.backward()
    torch.cuda.synchronize()
    return h_mid.detach(), W.detach(), [t.grad for t in leaves]


@pytest.mark.parametrize("name", ["f32_ragged", "bf16_tc", "bf16_small_like"])
def test_pallas_assemble_autograd_matches_oracle(name):
    from matrix_b200.assembly import pallas_assemble
    cfg, x, idx, alphas = _setup(name)
    h_mid, W, grads = _grads(pallas_assemble, cfg, x, idx, alphas)
    ref_h, ref_W, ref_g = _oracle(cfg, x, idx, alphas)
    tol = BF16_TOL if cfg.compute_dtype == "bfloat16" else F32_TOL
    assert_close(_np(h_mid), ref_h, tol, name="h_mid")
    assert_close(_np(W), ref_W, tol, name="W")
    for n, got, ref in zip(("g_gathered", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), grads, ref_g):
        assert got is not None, n
        assert_close(_np(got).reshape(np.shape(ref)), ref, tol, name=n)
    # dtypes follow the inputs, like jax.custom_vjp's cotangents
    assert grads[0].dtype == (torch.bfloat16 if cfg.bf16_pool else torch.float32)
    assert grads[5].shape == ()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("name", ["bf16_tc", "f32_ragged"])
def test_shard_pallas_assemble_on_a_nccl_group_equals_pallas_assemble(name):
    import torch.distributed as dist
    from matrix_b200.assembly import pallas_assemble, shard_pallas_assemble
    cfg, x, idx, alphas = _setup(name, seed=4)
    one = _grads(pallas_assemble, cfg, x, idx, alphas)
    started = False
    if not dist.is_initialized():
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                                device_id=torch.device("cuda", 0))
        started = True
    try:
        group = dist.new_group([0])
        sharded = _grads(lambda *a: shard_pallas_assemble(*a, mesh=group), cfg, x, idx, alphas)
    finally:
        if started:
            dist.destroy_process_group()
    for u, v in zip(one[:2], sharded[:2]):
        assert torch.equal(u, v)
    tol = BF16_TOL if cfg.compute_dtype == "bfloat16" else F32_TOL
    ref_h, ref_W, ref_g = _oracle(cfg, x, idx, alphas)
    for n, a, b, ref in zip(("g_gathered", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), one[2],
                            sharded[2], ref_g):
        # float atomics in g_alpha / g_W_base / g_b_base / g_gamma: equal up to their ordering
        assert_close(_np(b), _np(a), 1e-6, name=n)
        assert_close(_np(b).reshape(np.shape(ref)), ref, tol, name=n)


def test_cases_exist():
    assert {"f32_ragged", "bf16_tc", "bf16_small_like"} <= set(CASES)
