"""The RMSNorm restatement in the oracle: forward by definition (flax
nnx.RMSNorm: x * rsqrt(mean(x^2) + eps) * scale) and its VJP against central
finite differences in float64."""

from __future__ import annotations

import numpy as np

from oracle import dwa_oracle as O


def test_rms_norm_forward_definition():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 16))
    s = rng.standard_normal(16)
    y = O.rms_norm(x, s)
    ref = x / np.sqrt((x ** 2).mean(axis=1, keepdims=True) + 1e-6) * s
    np.testing.assert_allclose(y, ref, rtol=1e-14)
    # unit scale: every row has mean square 1 (up to eps)
    yn = O.rms_norm(x * 3.0, np.ones(16))
    np.testing.assert_allclose((yn ** 2).mean(axis=1), 1.0, rtol=1e-6)


def test_rms_norm_vjp_matches_finite_differences():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 8))
    s = rng.standard_normal(8)
    g = rng.standard_normal((3, 8))
    g_x, g_s = O.rms_norm_bwd(x, s, g)
    h = 1e-6

    def loss(xx, ss):
        return float(np.sum(O.rms_norm(xx, ss) * g))

    num_x = np.zeros_like(x)
    for idx in np.ndindex(*x.shape):
        e = np.zeros_like(x)
        e[idx] = h
        num_x[idx] = (loss(x + e, s) - loss(x - e, s)) / (2 * h)
    num_s = np.array([(loss(x, s + h * np.eye(8)[j]) - loss(x, s - h * np.eye(8)[j])) / (2 * h)
                      for j in range(8)])
    np.testing.assert_allclose(g_x, num_x, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(g_s, num_s, rtol=1e-6, atol=1e-9)
