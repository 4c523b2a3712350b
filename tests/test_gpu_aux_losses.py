"""Auxiliary losses (``dwa_aux_losses``) against the oracle's literal
restatement of losses.py:9-73 and its VJP (pinned by finite differences) in
float64, rtol 1e-5: a realistic shape with a row chosen by two queries, k = 1
(no pairs: l_div = 0), an alpha on the clip bound, the key gradient added into
a non-zero buffer, bit-identical repeats, and ``torch.autograd`` through
``aux_losses_with_grad``."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5
LAM = dict(lambda_util=0.01, lambda_div=0.01, lambda_norm=0.001, lambda_sparse=0.001)


def _case(B=8, k=32, S=4, N=20000, d_k=64, d=96, seed=0):
    rng = np.random.default_rng(seed)
    al = rng.random((B, k)).astype(np.float32) + 0.01
    al /= al.sum(-1, keepdims=True)
    idx = np.stack([rng.choice(N, size=k, replace=False) for _ in range(B)]).astype(np.int32)
    if B > 1 and k > 3:
        idx[1, 3] = idx[0, 0]
    soft = rng.random((B, N)).astype(np.float32)
    soft /= soft.sum(-1, keepdims=True)
    return dict(alphas=al, indices=idx, pool_keys=rng.standard_normal((S, N, d_k), dtype=np.float32),
                W=rng.standard_normal((B, d, d), dtype=np.float32) * 0.1,
                W_base=rng.standard_normal((d, d), dtype=np.float32) * 0.1, soft_full=soft)


def _dev(x):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in x.items()}


def _f64(x):
    return {k: (v.astype(np.float64) if v.dtype != np.int32 else v.astype(np.int64)) for k, v in x.items()}


@pytest.mark.parametrize("shape", [dict(), dict(B=3, k=1, N=500, d=32), dict(B=5, k=16, S=2, d_k=32, N=3000, d=64)])
def test_aux_losses_and_grads_match_oracle(shape):
    from matrix_b200.losses import aux_losses_and_grads
    x = _case(**shape)
    if x["alphas"].shape[1] > 1:
        x["alphas"][0, 0] = 1.0          # on the clip bound: half gradient
    d = _dev(x)
    # a non-zero buffer on the gradient's own scale (about 1e-7), so that adding
    # into it loses no bits to float32 rounding
    base = (np.random.default_rng(1).standard_normal(x["pool_keys"].shape) * 1e-7).astype(np.float32)
    gk = torch.from_numpy(base.copy()).cuda()
    losses, g = aux_losses_and_grads(**d, key_grad_into=gk, **LAM)
    torch.cuda.synchronize()
    ref = O.aux_losses(**_f64(x), **LAM)
    refg = O.aux_losses_bwd(**_f64(x), **LAM)
    for name in ("l_util", "l_div", "l_norm", "l_sparse", "total_aux"):
        r = float(ref[name])
        assert abs(float(losses[name]) - r) <= TOL * max(abs(r), 1e-3), f"{name}: {float(losses[name])} vs {r}"
    for name in ("g_alphas", "g_soft_full", "g_W", "g_W_base"):
        assert_close(g[name].cpu().numpy(), refg[name], TOL, name=name)
    assert_close(gk.cpu().numpy(), base.astype(np.float64) + refg["g_pool_keys"], TOL, name="g_pool_keys")


def test_repeats_are_bit_identical():
    from matrix_b200.losses import aux_losses_and_grads
    d = _dev(_case(seed=3))
    outs = []
    for _ in range(2):
        gk = torch.zeros_like(d["pool_keys"])
        losses, g = aux_losses_and_grads(**d, key_grad_into=gk, **LAM)
        outs.append(([float(v) for v in losses.values()], {k: v.cpu().numpy() for k, v in g.items()}, gk.cpu().numpy()))
    assert outs[0][0] == outs[1][0]
    for k in outs[0][1]:
        np.testing.assert_array_equal(outs[0][1][k], outs[1][1][k])
    np.testing.assert_array_equal(outs[0][2], outs[1][2])


def test_autograd_total_matches_explicit_grads():
    from matrix_b200.losses import aux_losses_and_grads, aux_losses_with_grad
    x = _case(seed=4)
    d = _dev(x)
    leaves = {k: d[k].clone().requires_grad_(True) for k in ("alphas", "soft_full", "W", "W_base", "pool_keys")}
    total, parts = aux_losses_with_grad(leaves["alphas"], d["indices"], leaves["pool_keys"], leaves["W"],
                                        leaves["W_base"], leaves["soft_full"], **LAM)
    (3.0 * total).backward()
    gk = torch.zeros_like(d["pool_keys"])
    _, g = aux_losses_and_grads(**d, key_grad_into=gk, **LAM)
    for k_ in ("alphas", "soft_full", "W", "W_base"):
        np.testing.assert_allclose(leaves[k_].grad.cpu().numpy(), 3.0 * g["g_" + k_].cpu().numpy(), rtol=1e-6)
    np.testing.assert_allclose(leaves["pool_keys"].grad.cpu().numpy(), 3.0 * gk.cpu().numpy(), rtol=1e-6)


@pytest.mark.parametrize("bounds,seqs", [([0, 9000, 20000], [0, 3, 8]), ([0, 7000, 7000, 20000], [0, 4, 4, 8])])
def test_sharded_aux_equals_single_call(bounds, seqs):
    """Ranks emulated on one GPU (rows and sequences split, an empty rank):
    the losses and g_alphas / g_W_base on every rank, and the ranks' slices of
    g_soft_full, g_W and the key gradient, equal the single call's."""
    from matrix_b200.losses import aux_losses_and_grads, sharded_aux_losses_and_grads
    x = _case(seed=5)
    d = _dev(x)
    gk_ref = torch.zeros_like(d["pool_keys"])
    ref, rg = aux_losses_and_grads(**d, key_grad_into=gk_ref, **LAM)
    world = len(bounds) - 1
    parts = [(bounds[r], bounds[r + 1], seqs[r], seqs[r + 1]) for r in range(world)]
    # phase 1 on every rank, then the sums, then phase 2 on every rank
    collected = []

    def run(r, reduce):
        lo, hi, s0, s1 = parts[r]
        gk = torch.zeros((d["pool_keys"].shape[0], hi - lo, d["pool_keys"].shape[2]), device="cuda")
        W_loc = d["W"][s0:s1].contiguous() if s1 > s0 else None
        out = sharded_aux_losses_and_grads(d["alphas"], d["indices"], d["pool_keys"][:, lo:hi].contiguous(), W_loc,
                                           d["W_base"], d["soft_full"][:, lo:hi].contiguous(), row_lo=lo,
                                           n_global=d["soft_full"].shape[1], key_grad_into=gk, reduce=reduce, **LAM)
        return out, gk

    def gather(part, rk, gwb):
        collected.append((part.clone(), rk.clone(), gwb.clone()))
        return part, rk, gwb

    for r in range(world):          # phase 1 only: record every rank's partials
        run(r, gather)
    sums = [sum(c[i] for c in collected) for i in range(3)]
    results = [run(r, lambda p, rk, g: tuple(t.clone() for t in sums)) for r in range(world)]
    torch.cuda.synchronize()
    for (losses, g), gk in results:
        for name in ("l_util", "l_div", "l_norm", "l_sparse", "total_aux"):
            r_ = float(ref[name])
            assert abs(float(losses[name]) - r_) <= TOL * max(abs(r_), 1e-3), name
        assert_close(g["g_alphas"].cpu().numpy(), rg["g_alphas"].cpu().numpy(), TOL, name="g_alphas")
        assert_close(g["g_W_base"].cpu().numpy(), rg["g_W_base"].cpu().numpy(), TOL, name="g_W_base")
    assert_close(np.concatenate([g["g_soft_full"].cpu().numpy() for (_, g), _ in results], axis=1),
                 rg["g_soft_full"].cpu().numpy(), TOL, name="g_soft_full")
    assert_close(np.concatenate([g["g_W"].cpu().numpy() for (_, g), _ in results], axis=0),
                 rg["g_W"].cpu().numpy(), TOL, name="g_W")
    assert_close(np.concatenate([gk.cpu().numpy() for _, gk in results], axis=1), gk_ref.cpu().numpy(), TOL,
                 name="g_pool_keys")
