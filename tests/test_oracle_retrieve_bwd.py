"""The oracle's retrieval VJP (``retrieve_bwd``) against central differences of
the oracle's own forward (``retrieve``, pinned to the reference by golden
vectors) in float64: for ``L = Σ g_α·α + Σ g_soft·soft_full``, every
parameter the reference trains through retrieval (``z``, ``W_Q``,
``aspect_weights``, ``tau``) and the key cache, in warmup and gate mode, with
IVF and full search.  The selection is checked to stay put under the
perturbation (no index flips), so the difference quotient is the derivative.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import dwa_oracle as O

H = 1e-6


def _case(seed, use_ivf):
    rng = np.random.default_rng(seed)
    B, S, d_k, d_A, C, N = 3, 2, 8, 12, 6, 120
    x = dict(
        z=rng.standard_normal((B, d_A)),
        W_Q=rng.standard_normal((S, d_k, d_A)) * d_A ** -0.5,
        aspect_weights=rng.standard_normal(S) * 0.3,
        tau=np.float64(0.05),
        centroids=rng.standard_normal((S, C, d_k)),
        pool_keys=rng.standard_normal((S, N, d_k)),
    )
    kw = dict(k=5, m=2, T=0.7, use_ivf=use_ivf, tie_break="index")
    g_alphas = rng.standard_normal((B, 5))
    g_soft = rng.standard_normal((B, N)) * 0.5
    return x, kw, g_alphas, g_soft


def _loss(x, kw, lam, warm, g_alphas, g_soft):
    a, idx, sf = O.retrieve(x["z"], x["W_Q"], x["aspect_weights"], x["tau"], x["centroids"],
                            x["pool_keys"], lambda_val=lam, is_warmup=warm, **kw)
    return float(np.sum(g_alphas * a) + np.sum(g_soft * sf)), idx


@pytest.mark.parametrize("use_ivf", [True, False])
@pytest.mark.parametrize("warm,lam", [(True, 1.0), (False, 5.0), (False, -2.0)])
def test_retrieve_bwd_matches_finite_differences(use_ivf, warm, lam):
    x, kw, g_alphas, g_soft = _case(7 if use_ivf else 9, use_ivf)
    g = O.retrieve_bwd(x["z"], x["W_Q"], x["aspect_weights"], x["tau"], x["centroids"], x["pool_keys"],
                       lambda_val=lam, is_warmup=warm, g_alphas=g_alphas, g_soft_full=g_soft, **kw)
    _, idx0 = _loss(x, kw, lam, warm, g_alphas, g_soft)
    rng = np.random.default_rng(3)
    names = {"z": "g_z", "W_Q": "g_W_Q", "aspect_weights": "g_aspect_weights", "tau": "g_tau",
             "pool_keys": "g_pool_keys"}
    for name, gname in names.items():
        if warm and name == "tau":
            assert g[gname] == 0.0
            continue
        arr = np.asarray(x[name], dtype=np.float64)
        flat_n = arr.size
        picks = rng.choice(flat_n, size=min(8, flat_n), replace=False) if flat_n > 1 else [0]
        for p in picks:
            vals = []
            for sgn in (1.0, -1.0):
                y = dict(x)
                pert = arr.copy().reshape(-1)
                pert[p] += sgn * H
                y[name] = pert.reshape(arr.shape) if arr.ndim else np.float64(pert[0])
                L, idx = _loss(y, kw, lam, warm, g_alphas, g_soft)
                np.testing.assert_array_equal(idx, idx0)
                vals.append(L)
            fd = (vals[0] - vals[1]) / (2 * H)
            an = np.asarray(g[gname], dtype=np.float64).reshape(-1)[p]
            scale = max(1e-3, float(np.max(np.abs(g[gname]))))
            assert abs(fd - an) <= 1e-6 * scale, f"{name}[{p}]: fd {fd} analytic {an}"


def test_retrieve_bwd_separates_the_two_cotangents():
    """The VJP is linear in (g_α, g_soft): each alone sums to both together."""
    x, kw, g_alphas, g_soft = _case(11, True)
    args = (x["z"], x["W_Q"], x["aspect_weights"], x["tau"], x["centroids"], x["pool_keys"])
    both = O.retrieve_bwd(*args, lambda_val=5.0, is_warmup=False, g_alphas=g_alphas, g_soft_full=g_soft, **kw)
    a = O.retrieve_bwd(*args, lambda_val=5.0, is_warmup=False, g_alphas=g_alphas, **kw)
    s = O.retrieve_bwd(*args, lambda_val=5.0, is_warmup=False, g_soft_full=g_soft, **kw)
    for key in ("g_z", "g_W_Q", "g_aspect_weights", "g_pool_keys"):
        np.testing.assert_allclose(both[key], a[key] + s[key], rtol=1e-12, atol=1e-14)
