"""The oracle's auxiliary-loss VJP (``aux_losses_bwd``) against central
differences of its ``aux_losses`` (a literal restatement of losses.py:9-73) in
float64, including repeated indices (one pool row chosen twice) and an alpha
exactly on the clip bound (jnp.clip's half gradient)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import dwa_oracle as O

LAM = dict(lambda_util=0.01, lambda_div=0.01, lambda_norm=0.001, lambda_sparse=0.001)


def _case(seed=0):
    rng = np.random.default_rng(seed)
    B, k, S, N, d_k, d = 3, 5, 2, 40, 6, 4
    al = rng.random((B, k)) + 0.05
    al = al / al.sum(-1, keepdims=True)
    idx = rng.integers(0, N, size=(B, k))
    idx[1, 2] = idx[0, 0]
    soft = rng.random((B, N))
    soft = soft / soft.sum(-1, keepdims=True)
    return dict(alphas=al, indices=idx, pool_keys=rng.standard_normal((S, N, d_k)),
                W=rng.standard_normal((B, d, d)), W_base=rng.standard_normal((d, d)), soft_full=soft)


def test_aux_bwd_matches_finite_differences():
    x = _case()
    g = O.aux_losses_bwd(**x, **LAM)
    h = 1e-6
    rng = np.random.default_rng(1)
    for name, gname in (("alphas", "g_alphas"), ("soft_full", "g_soft_full"), ("W", "g_W"),
                        ("W_base", "g_W_base"), ("pool_keys", "g_pool_keys")):
        arr = x[name]
        for p in rng.choice(arr.size, size=min(10, arr.size), replace=False):
            vals = []
            for sgn in (1.0, -1.0):
                y = dict(x)
                a = arr.copy().reshape(-1)
                a[p] += sgn * h
                y[name] = a.reshape(arr.shape)
                vals.append(float(O.aux_losses(**y, **LAM)["total_aux"]))
            fd = (vals[0] - vals[1]) / (2 * h)
            an = float(g[gname].reshape(-1)[p])
            assert abs(fd - an) <= 1e-7 + 1e-6 * abs(an), f"{name}[{p}]: fd {fd} analytic {an}"


def test_aux_bwd_duplicate_rows_accumulate_and_clip_bound():
    x = _case(2)
    x["alphas"][2] = np.array([1.0, 0.0, 0.0, 0.0, 0.0])
    g = O.aux_losses_bwd(**x, **LAM)
    B = x["alphas"].shape[0]
    assert g["g_alphas"][2, 0] == pytest.approx(-0.001 * (np.log(1.0) + 1) / B * 0.5)
    assert (g["g_alphas"][2, 1:] == 0).all()
    # the doubly chosen row receives both contributions
    r = x["indices"][0, 0]
    assert np.abs(g["g_pool_keys"][:, r]).sum() > 0
