"""Parity of the CUDA assembly (forward + custom VJP) with the oracle and with
golden vectors produced by the reference's own source.

Tolerances (north-star): float32 activations rtol 1e-5, bfloat16 rtol 2e-2,
each with an absolute floor of rtol * max|expected| (``assert_close``).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close, load_golden
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F32_TOL, BF16_TOL = 1e-5, 2e-2


def _cfg(d, r, k, N, dtype, C=16, D=None):
    return DWAConfig(D=D or d * (2 * r + 1), N=N, use_ivf=True, C=C, m=2, d_A=d, d_B=d, r=r,
                     k_max=k, S=4, d_k=64, T=1.0, gamma_init=0.1,
                     bf16_pool=(dtype == "bfloat16"), compute_dtype=dtype)


# name -> (cfg, B, T)
CASES = {
    "f32_refsmall": (DWAConfig(D=2048, N=512, C=128, m=8, d_A=64, d_B=64, r=4, k_max=8, S=2,
                               d_k=32, gamma_init=0.01, bf16_pool=False), 4, 64),
    "f32_ragged": (_cfg(96, 8, 12, 600, "float32", C=24, D=1640), 10, 40),
    "bf16_tc": (_cfg(256, 8, 16, 512, "bfloat16"), 3, 200),
    "bf16_small_like": (_cfg(1024, 8, 32, 512, "bfloat16"), 8, 256),
    "bf16_ragged": (_cfg(96, 8, 12, 600, "bfloat16", C=24, D=1640), 5, 40),
    # 19 x 32 tiles of W (four waves and more on 148 SMs): the W GEMM whose
    # epilogue moves W_base, W and W_act by TMA; square, then with partial
    # 32 x 32 boxes at the edges (d 1000)
    "bf16_w_tma": (_cfg(1024, 8, 8, 64, "bfloat16"), 19, 32),
    "bf16_w_tma_edges": (_cfg(1000, 8, 8, 64, "bfloat16"), 19, 24),
}


def _setup(name, seed=11, zero_alpha=False):
    cfg, B, T = CASES[name]
    x = make_inputs(cfg, B, T, seed, variant="rich")
    rng = np.random.default_rng(seed + 1)
    idx = np.stack([rng.choice(cfg.N, cfg.k_max, replace=False) for _ in range(B)]).astype(np.int32)
    a = rng.standard_normal((B, cfg.k_max))
    alphas = np.exp(a) / np.exp(a).sum(-1, keepdims=True)
    if zero_alpha:
        alphas[:] = 0
    return cfg, x, idx, alphas.astype(np.float32)


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def _oracle(cfg, x, idx, alphas):
    f = np.float64
    gathered = x.pool[idx].astype(f)
    h_mid, W = O.assemble(gathered, alphas.astype(f), x.h_A.astype(f), x.W_base.astype(f),
                          x.b_base.astype(f), f(x.gamma), cfg.d_B, cfg.r, cfg.d_A)
    grads = O.assemble_bwd(gathered, alphas.astype(f), x.h_A.astype(f), W, f(x.gamma),
                           x.g_hmid.astype(f), x.g_W.astype(f), cfg.d_B, cfg.r, cfg.d_A)
    return h_mid, W, grads


def _run(cfg, x, idx, alphas, fused):
    from matrix_b200.assembly import assemble_backward, assemble_forward
    act = torch.bfloat16 if cfg.compute_dtype == "bfloat16" else torch.float32
    pool_dt = torch.bfloat16 if cfg.bf16_pool else torch.float32
    pool = _dev(x.pool, pool_dt)
    idx_t = _dev(idx)
    rows = pool if fused else pool[idx_t.long()].contiguous()
    ri = idx_t if fused else None
    h_A = _dev(x.h_A, act)
    args = (_dev(alphas), h_A, _dev(x.W_base), _dev(x.b_base), torch.tensor(x.gamma).cuda())
    h_mid, W, W_act = assemble_forward(rows, *args, cfg.d_B, cfg.r, cfg.d_A, row_index=ri)
    grads = assemble_backward(rows, args[0], h_A, W_act, args[4], _dev(x.g_hmid, act),
                              _dev(x.g_W), cfg.d_B, cfg.r, cfg.d_A, row_index=ri)
    torch.cuda.synchronize()
    return h_mid, W, grads


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("fused", [False, True])
def test_forward_backward_match_oracle(name, fused):
    from matrix_b200 import _lib
    from matrix_b200.runtime import raise_on_device_status
    cfg, x, idx, alphas = _setup(name)
    before = _lib.launch_counters()
    h_mid, W, grads = _run(cfg, x, idx, alphas, fused)
    after = _lib.launch_counters()
    raise_on_device_status()
    ref_h, ref_W, ref_g = _oracle(cfg, x, idx, alphas)
    tol = BF16_TOL if cfg.compute_dtype == "bfloat16" else F32_TOL
    assert_close(_np(h_mid), ref_h, tol, name="h_mid")
    assert_close(_np(W), ref_W, tol, name="W")
    names = ("g_rows", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma")
    for n, got, ref in zip(names, grads, ref_g):
        assert_close(_np(got).reshape(np.shape(ref)), ref, tol, name=n)
    if cfg.compute_dtype == "bfloat16" and cfg.d_A % 64 == 0:
        assert after[1] > before[1], "bf16 GEMMs did not run on the tensor cores"


@pytest.mark.parametrize("name", ["bf16_tc", "f32_ragged"])
def test_fused_gather_equals_gathered_rows(name):
    cfg, x, idx, alphas = _setup(name, seed=3)
    a = _run(cfg, x, idx, alphas, fused=False)
    b = _run(cfg, x, idx, alphas, fused=True)
    # h_mid, W, g_rows, g_hA have a fixed summation order: bit-identical.
    for u, v in zip((a[0], a[1], a[2][0], a[2][2]), (b[0], b[1], b[2][0], b[2][2])):
        assert torch.equal(u, v)
    # g_alpha, g_W_base, g_b_base, g_gamma are accumulated with float atomics
    for u, v in zip((a[2][1], *a[2][3:]), (b[2][1], *b[2][3:])):
        assert_close(_np(u), _np(v), 1e-6)


@pytest.mark.parametrize("name", ["bf16_tc", "f32_refsmall"])
def test_zero_alphas_give_base(name):
    cfg, x, idx, alphas = _setup(name, zero_alpha=True)
    h_mid, W, _ = _run(cfg, x, idx, alphas, fused=True)
    np.testing.assert_allclose(_np(W), np.broadcast_to(x.W_base, _np(W).shape), rtol=0, atol=1e-6)


@pytest.mark.parametrize("case", ["smoke", "refsmall", "ragged"])
def test_assembly_matches_reference_golden(case):
    """The fp32 kernels against outputs of the reference's own assemble_jax /
    _pallas_assemble_bwd (tests/golden/make_golden.py)."""
    from test_oracle_golden import _inputs
    cfg, x, _, _ = _inputs(case)
    g = load_golden(case)
    import dataclasses
    cfg = dataclasses.replace(cfg, bf16_pool=False)
    h_mid, W, grads = _run(cfg, x, g["gate_indices"].astype(np.int32), g["gate_alphas"], True)
    assert_close(_np(h_mid), g["h_mid"], F32_TOL, name="h_mid")
    assert_close(_np(W), g["W"], F32_TOL, name="W")
    for n, got in zip(("g_gathered", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"), grads):
        assert_close(_np(got).reshape(g[n].shape), g[n], 2e-5, name=n)


def test_autograd_function_matches_explicit_backward():
    from matrix_b200.assembly import pallas_assemble
    cfg, x, idx, alphas = _setup("bf16_tc", seed=5)
    gathered = _dev(x.pool[idx], torch.float32).requires_grad_(True)
    al = _dev(alphas).requires_grad_(True)
    h_A = _dev(x.h_A, torch.bfloat16).requires_grad_(True)
    W_base = _dev(x.W_base).requires_grad_(True)
    b_base = _dev(x.b_base).requires_grad_(True)
    gamma = torch.tensor(x.gamma, device="cuda").requires_grad_(True)
    h_mid, W = pallas_assemble(gathered, al, h_A, W_base, b_base, gamma, cfg.d_B, cfg.r, cfg.d_A)
    g_h, g_W = _dev(x.g_hmid, torch.bfloat16), _dev(x.g_W)
    grads = torch.autograd.grad((h_mid, W), (gathered, al, h_A, W_base, b_base, gamma), (g_h, g_W))
    ref_h, ref_W, ref_g = _oracle(cfg, x, idx, alphas)
    assert gamma.grad is None and grads[5].shape == gamma.shape
    for got, ref in zip(grads, ref_g):
        assert_close(_np(got).reshape(np.shape(ref)), ref, BF16_TOL)


def test_bad_row_index_sets_status_bit():
    from matrix_b200.assembly import assemble_forward
    from matrix_b200.runtime import workspace_status
    cfg, x, idx, alphas = _setup("bf16_tc")
    idx = idx.copy()
    idx[1, 3] = cfg.N + 5          # outside the pool: the row reads as zeros, status flags it
    workspace_status(clear=True)
    pool = _dev(x.pool, torch.bfloat16)
    h_mid, W, _ = assemble_forward(pool, _dev(alphas), _dev(x.h_A, torch.bfloat16),
                                   _dev(x.W_base), _dev(x.b_base), torch.tensor(x.gamma).cuda(),
                                   cfg.d_B, cfg.r, cfg.d_A, row_index=_dev(idx))
    st = workspace_status(clear=True)
    assert any(v & 0x1 for v in st.values())
    assert torch.isfinite(h_mid.float()).all()
