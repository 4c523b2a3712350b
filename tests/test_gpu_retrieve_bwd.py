"""Retrieval VJP (``dwa_retrieve_bwd``) against the oracle's ``retrieve_bwd``
in float64 (itself pinned by finite differences of the oracle forward), rtol
1e-5 of each gradient's largest entry:

* IVF on Zipf lists in warmup, gate (lambda 5) and gate with lambda < 0 (the
  selection ranks the gate term), with both cotangents, with g_alphas alone
  (the key pass visits only the probed lists' tiles) and with g_soft_full
  alone; the key-cache gradient;
* full search (every row a candidate);
* 40 queries (two key passes of at most 32) and a bf16 z;
* bit-identical repeats, and ``torch.autograd`` through
  ``MultiAspectRetrieval`` giving the same gradients as the explicit call.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _setup(B=6, seed=8, use_ivf=True):
    cfg = DWAConfig(D=17 * 64, N=41 * 487, use_ivf=use_ivf, C=41, m=5, d_A=64, d_B=64, r=8, k_max=24,
                    S=4, d_k=64, T=0.8, gamma_init=0.1, bf16_pool=False)
    x = make_inputs(cfg, B, 16, seed, variant="rich", zipf=1.1)
    rng = np.random.default_rng(seed + 100)
    g_alphas = rng.standard_normal((B, cfg.k_max)).astype(np.float32)
    g_soft = (rng.standard_normal((B, cfg.N)) * 50.0).astype(np.float32)
    return cfg, x, g_alphas, g_soft


def _run(cfg, x, lam, warm, g_alphas, g_soft, want_keys, z_dtype=None):
    from matrix_b200.retrieval import retrieve, retrieve_backward
    off = x.list_offsets if cfg.use_ivf else None
    max_list = int(np.diff(off).max()) if cfg.use_ivf else None
    z = _dev(x.z) if z_dtype is None else _dev(x.z).to(z_dtype)
    args = (z, _dev(x.W_Q), _dev(x.aspect_weights), torch.tensor(x.tau).cuda(), _dev(x.centroids),
            _dev(x.keys), lam, warm)
    kw = dict(k=cfg.k_max, m=cfg.m, T=cfg.T, use_ivf=cfg.use_ivf,
              list_offsets=_dev(off) if off is not None else None, max_list=max_list)
    a, i, sf = retrieve(*args, **kw, want_soft_full=True)
    g = retrieve_backward(*args, a, i, sf, None if g_alphas is None else _dev(g_alphas),
                          None if g_soft is None else _dev(g_soft), **kw, want_key_grad=want_keys)
    torch.cuda.synchronize()
    return {k_: (v.cpu().numpy() if v is not None else None) for k_, v in g.items()}, i.cpu().numpy()


def _oracle(cfg, x, lam, warm, g_alphas, g_soft, z=None):
    f = np.float64
    return O.retrieve_bwd((x.z if z is None else z).astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f),
                          f(x.tau), x.centroids.astype(f), x.keys.astype(f), k=cfg.k_max, m=cfg.m, T=cfg.T,
                          lambda_val=lam, is_warmup=warm,
                          g_alphas=None if g_alphas is None else g_alphas.astype(f),
                          g_soft_full=None if g_soft is None else g_soft.astype(f), use_ivf=cfg.use_ivf,
                          list_offsets=x.list_offsets if cfg.use_ivf else None, tie_break="index")


def _check(got, ref, tag, keys=False):
    for name in ("g_z", "g_W_Q", "g_aspect_weights"):
        assert_close(got[name], ref[name], TOL, name=f"{name} {tag}")
    assert_close(np.array([got["g_tau"]]).reshape(1), np.array([ref["g_tau"]]).reshape(1), TOL,
                 atol_scale=max(abs(float(ref["g_tau"])), 1e-3), name=f"g_tau {tag}")
    if keys:
        assert_close(got["g_pool_keys"], ref["g_pool_keys"], TOL, name=f"g_pool_keys {tag}")


@pytest.mark.parametrize("warm,lam", [(True, 1.0), (False, 5.0), (False, -2.0)])
@pytest.mark.parametrize("which", ["both", "alphas", "soft"])
def test_ivf_vjp_matches_oracle(warm, lam, which):
    cfg, x, ga, gs = _setup()
    ga = ga if which in ("both", "alphas") else None
    gs = gs if which in ("both", "soft") else None
    got, _ = _run(cfg, x, lam, warm, ga, gs, want_keys=False)
    _check(got, _oracle(cfg, x, lam, warm, ga, gs), f"warm={warm} lam={lam} {which}")


@pytest.mark.parametrize("warm,lam", [(True, 1.0), (False, 5.0)])
def test_key_cache_gradient_matches_oracle(warm, lam):
    cfg, x, ga, gs = _setup(B=5, seed=9)
    got, _ = _run(cfg, x, lam, warm, ga, gs, want_keys=True)
    _check(got, _oracle(cfg, x, lam, warm, ga, gs), f"keys warm={warm}", keys=True)


@pytest.mark.parametrize("warm,lam", [(True, 1.0), (False, 5.0)])
def test_full_search_vjp_matches_oracle(warm, lam):
    cfg, x, ga, gs = _setup(B=4, seed=10, use_ivf=False)
    got, _ = _run(cfg, x, lam, warm, ga, gs, want_keys=True)
    _check(got, _oracle(cfg, x, lam, warm, ga, gs), f"full warm={warm}", keys=True)


def test_forty_queries_and_bf16_z():
    from matrix_b200.synthetic import bf16_round
    cfg, x, ga, gs = _setup(B=40, seed=12)
    got, _ = _run(cfg, x, 5.0, False, ga, gs, want_keys=False)
    _check(got, _oracle(cfg, x, 5.0, False, ga, gs), "B=40")
    x.z = bf16_round(x.z)
    got, _ = _run(cfg, x, 5.0, False, ga, gs, want_keys=False, z_dtype=torch.bfloat16)
    _check(got, _oracle(cfg, x, 5.0, False, ga, gs), "bf16 z")


def test_repeats_are_bit_identical():
    cfg, x, ga, gs = _setup(B=7, seed=13)
    g1, _ = _run(cfg, x, 5.0, False, ga, gs, want_keys=True)
    g2, _ = _run(cfg, x, 5.0, False, ga, gs, want_keys=True)
    for name in g1:
        np.testing.assert_array_equal(g1[name], g2[name], err_msg=name)


def test_autograd_through_module_matches_explicit_vjp():
    from matrix_b200.retrieval import MultiAspectRetrieval
    cfg, x, ga, gs = _setup(B=5, seed=14)
    mod = MultiAspectRetrieval(cfg, device="cuda")
    mod.W_Q = _dev(x.W_Q).requires_grad_(True)
    mod.aspect_weights = _dev(x.aspect_weights).requires_grad_(True)
    mod.tau = torch.tensor(x.tau).cuda().requires_grad_(True)
    mod.centroids = _dev(x.centroids)
    mod.set_lists(_dev(x.list_offsets), int(np.diff(x.list_offsets).max()))
    z = _dev(x.z).requires_grad_(True)
    keys = _dev(x.keys)
    a, i, sf = mod(z, keys, 5.0, False)
    loss = (a * _dev(ga)).sum() + (sf * _dev(gs)).sum()
    loss.backward()
    got, _ = _run(cfg, x, 5.0, False, ga, gs, want_keys=False)
    np.testing.assert_array_equal(z.grad.cpu().numpy(), got["g_z"])
    np.testing.assert_array_equal(mod.W_Q.grad.cpu().numpy(), got["g_W_Q"])
    np.testing.assert_array_equal(mod.aspect_weights.grad.cpu().numpy(), got["g_aspect_weights"])
    np.testing.assert_array_equal(mod.tau.grad.cpu().numpy(), got["g_tau"])
