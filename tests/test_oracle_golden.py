"""Pin the NumPy oracle to golden vectors made by executing the reference's own
source (``tests/golden/make_golden.py``) and to the invariants the reference's
tests assert (tests/test_retrieval.py:48-97, tests/test_assembly.py:38-95).
CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close, load_golden
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O

import importlib.util
import os

_spec = importlib.util.spec_from_file_location(
    "make_golden_cases", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))


def _cases():
    # Read the CASES table without importing the reference: parse the module
    # source up to the table only by executing it with a dummy numpy_jax.
    import ast
    src = open(_spec.origin).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.Assign) and getattr(node.targets[0], "id", "") == "CASES":
            ns = {"WORKLOADS": __import__("matrix_b200.config", fromlist=["WORKLOADS"]).WORKLOADS}
            return eval(compile(ast.Expression(node.value), "CASES", "eval"), ns)
    raise RuntimeError("CASES not found")


CASES = _cases()


def _inputs(name, dtype=np.float64):
    kw, B, seq, seed, variant, modes, with_asm = CASES[name]
    cfg = DWAConfig(**kw)
    x = make_inputs(cfg, B, seq, seed, variant=variant)
    return cfg, x, modes, with_asm


@pytest.mark.parametrize("name", list(CASES))
def test_inputs_regenerate_identically(name):
    _, x, _, _ = _inputs(name)
    g = load_golden(name)
    assert str(g["digest"]) == x.digest()


def _boundary_gap(scores, k):
    s = np.sort(scores)[::-1]
    return s[k - 1] - s[k] if len(s) > k else np.inf


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_retrieval_matches_golden(name, dtype):
    cfg, x, modes, _ = _inputs(name)
    g = load_golden(name)
    for is_warmup, lam in modes:
        tag = "warmup" if is_warmup else "gate"
        c = lambda a: np.asarray(a, dtype=dtype)  # noqa: E731
        alphas, indices, soft_full, internals = O.retrieve(
            c(x.z), c(x.W_Q), c(x.aspect_weights), dtype(x.tau), c(x.centroids), c(x.keys),
            k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam, is_warmup=is_warmup,
            return_internals=True)
        # indices bit-exact wherever the k-th / (k+1)-th score gap is resolvable
        for b in range(indices.shape[0]):
            gap = _boundary_gap(internals["s_i"][b], cfg.k_max)
            assert gap > 1e-6, f"{name}/{tag} b={b}: seed has a near-tie at the top-k boundary"
        np.testing.assert_array_equal(indices, g[f"{tag}_indices"])
        tol = 1e-5 if dtype == np.float32 else 2e-6
        assert_close(alphas, g[f"{tag}_alphas"], tol, name=f"{name}/{tag}/alphas")
        assert_close(soft_full, g[f"{tag}_soft_full"], tol, name=f"{name}/{tag}/soft_full")


@pytest.mark.parametrize("name", [n for n in CASES if CASES[n][6]])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_assembly_matches_golden(name, dtype):
    cfg, x, _, _ = _inputs(name)
    g = load_golden(name)
    c = lambda a: np.asarray(a, dtype=dtype)  # noqa: E731
    gathered = O.gather(c(x.pool), g["gate_indices"], out_dtype=dtype)
    alphas = c(g["gate_alphas"])
    gamma = dtype(x.gamma)
    h_mid, W = O.assemble(gathered, alphas, c(x.h_A), c(x.W_base), c(x.b_base), gamma,
                          cfg.d_B, cfg.r, cfg.d_A)
    tol = 1e-5
    assert_close(h_mid, g["h_mid"], tol, name="h_mid")
    assert_close(W, g["W"], tol, name="W")
    # The Pallas kernel body computes the same values; rows a B % 8 tail leaves
    # unwritten are NaN in the golden (assembly_pallas.py:100,131).
    B = h_mid.shape[0]
    written = B if B <= 8 else B - B % 8
    pal = O.pallas_forward(gathered, alphas, c(x.h_A), c(x.W_base), c(x.b_base), gamma,
                           cfg.d_B, cfg.r, cfg.d_A)
    assert_close(pal[:written], g["h_mid_pallas"][:written], tol, name="h_mid_pallas")
    assert np.isnan(g["h_mid_pallas"][written:]).all()
    grads = O.assemble_bwd(gathered, alphas, c(x.h_A), W, gamma, c(x.g_hmid), c(x.g_W),
                           cfg.d_B, cfg.r, cfg.d_A)
    for gname, got in zip(("g_gathered", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"),
                          grads):
        assert_close(got, g[gname], 2e-5, name=gname)
    s3 = cfg.factor_split[2]
    assert not np.any(grads[0][:, :, s3:]), "pad columns of g_gathered must be zero"


# --- invariants asserted by the reference's own tests ----------------------

@pytest.fixture(scope="module")
def refsmall():
    return _inputs("refsmall")


def test_alphas_sum_to_one_and_nonnegative(refsmall):
    cfg, x, modes, _ = refsmall
    for is_warmup, lam in modes:
        a, idx, sf = O.retrieve(x.z, x.W_Q, x.aspect_weights, x.tau, x.centroids, x.keys,
                                k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam,
                                is_warmup=is_warmup)
        assert np.allclose(a.sum(-1), 1.0, atol=1e-5)          # test_retrieval.py:49-53
        assert (a >= 0).all()                                    # :55-58
        assert ((idx >= 0) & (idx < cfg.N)).all()                # :60-64
        assert np.allclose(sf.sum(-1), 1.0, atol=1e-4)           # :66-70


def test_zero_alphas_give_base_and_passthrough(refsmall):
    cfg, x, _, _ = refsmall
    g = load_golden("refsmall")
    gathered = O.gather(x.pool, g["gate_indices"])
    zero = np.zeros_like(g["gate_alphas"])
    _, W = O.assemble(gathered, zero, x.h_A, x.W_base, x.b_base, x.gamma, cfg.d_B, cfg.r, cfg.d_A)
    assert np.allclose(W, x.W_base[None], atol=1e-6)            # test_assembly.py:38-45
    h_mid, _ = O.assemble(gathered, zero, x.h_A, np.zeros_like(x.W_base),
                          np.zeros_like(x.b_base), 0.0, cfg.d_B, cfg.r, cfg.d_A)
    assert np.allclose(h_mid, x.h_A, atol=1e-6)                 # :47-56


def test_batch_independence(refsmall):
    cfg, x, _, _ = refsmall
    g = load_golden("refsmall")
    gathered = O.gather(x.pool, g["gate_indices"])
    a = g["gate_alphas"]
    full, _ = O.assemble(gathered, a, x.h_A, x.W_base, x.b_base, x.gamma, cfg.d_B, cfg.r, cfg.d_A)
    one, _ = O.assemble(gathered[:1], a[:1], x.h_A[:1], x.W_base, x.b_base, x.gamma,
                        cfg.d_B, cfg.r, cfg.d_A)
    assert np.allclose(full[:1], one, atol=1e-5)                # :88-95


def test_backward_is_the_gradient_of_the_forward():
    """The analytic VJP (assembly_pallas.py:246-329) equals central differences of
    ``assemble_jax`` (the contract ``jax.grad(assemble_jax) == _pallas_assemble_bwd``)."""
    rng = np.random.default_rng(5)
    B, k, d, r, T = 2, 3, 6, 2, 5
    D = d * r * 2 + d + 3
    gathered = rng.standard_normal((B, k, D))
    alphas = rng.random((B, k))
    h_A = rng.standard_normal((B, T, d))
    W_base = rng.standard_normal((d, d)) * 0.1
    b_base = rng.standard_normal(d) * 0.1
    gamma = 0.3
    g_h = rng.standard_normal((B, T, d))
    g_W = rng.standard_normal((B, d, d))

    def loss(gathered, alphas, h_A, W_base, b_base, gamma):
        h, W = O.assemble(gathered, alphas, h_A, W_base, b_base, gamma, d, r, d)
        return float(np.sum(h * g_h) + np.sum(W * g_W))

    args = [gathered, alphas, h_A, W_base, b_base, np.array(gamma)]
    _, W = O.assemble(*args[:5], gamma, d, r, d)
    grads = O.assemble_bwd(gathered, alphas, h_A, W, gamma, g_h, g_W, d, r, d)
    eps = 1e-6
    for i, (arg, g) in enumerate(zip(args, grads)):
        num = np.zeros_like(arg, dtype=np.float64)
        flat = arg.reshape(-1)
        for j in range(flat.size):
            old = flat[j]
            flat[j] = old + eps
            lp = loss(*args[:5], float(args[5]))
            flat[j] = old - eps
            lm = loss(*args[:5], float(args[5]))
            flat[j] = old
            num.reshape(-1)[j] = (lp - lm) / (2 * eps)
        assert_close(g, num, 1e-6, name=f"grad[{i}]")


def test_csr_lists_reduce_to_equal_lists():
    cfg, x, modes, _ = _inputs("refsmall")
    off = O.equal_list_offsets(cfg.N, cfg.C)
    for is_warmup, lam in modes:
        a1, i1, s1 = O.retrieve(x.z, x.W_Q, x.aspect_weights, x.tau, x.centroids, x.keys,
                                k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam, is_warmup=is_warmup)
        a2, i2, s2 = O.retrieve(x.z, x.W_Q, x.aspect_weights, x.tau, x.centroids, x.keys,
                                k=cfg.k_max, m=cfg.m, T=cfg.T, lambda_val=lam,
                                is_warmup=is_warmup, list_offsets=off, tie_break="index")
        np.testing.assert_array_equal(i1, i2)
        np.testing.assert_array_equal(a1, a2)
