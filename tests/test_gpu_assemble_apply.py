"""Parity of ``dwa_assemble_apply`` (h_mid only, the Pallas kernel's factored
form, src/dwa/assembly_pallas.py:85-132) with the oracle's ``assemble_jax``
restatement, and with a plain PyTorch fp32 statement at the decode shape
(d 4096, one to five rows per sequence, up to 128 retrieved rows).

Tolerances as for the forward: float32 activations rtol 1e-5, bfloat16 rtol
2e-2, each with an absolute floor of rtol * max|expected| (``assert_close``).
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

F32_TOL, BF16_TOL = 1e-5, 2e-2


def _cfg(d, r, k, N, dtype, C=16, D=None):
    return DWAConfig(D=D or d * (2 * r + 1), N=N, use_ivf=True, C=C, m=2, d_A=d, d_B=d, r=r,
                     k_max=k, S=4, d_k=64, T=1.0, gamma_init=0.1,
                     bf16_pool=(dtype == "bfloat16"), compute_dtype=dtype)


# name -> (cfg, B, T); T <= 16 runs the factored kernels, T = 40 the W path;
# B*T <= 16 the row kernel for the base product, above it a GEMM
CASES = {
    "f32_decode": (_cfg(256, 8, 16, 512, "float32"), 5, 1),
    "bf16_decode": (_cfg(1024, 8, 32, 512, "bfloat16"), 8, 1),
    "bf16_t3_pad": (_cfg(96, 8, 12, 600, "bfloat16", C=24, D=1640), 5, 3),
    "f32_t16_r4": (_cfg(64, 4, 8, 512, "float32"), 3, 16),
    "f32_odd_dims": (_cfg(60, 3, 5, 600, "float32", C=24, D=60 * 7 + 2), 2, 2),
    "bf16_b24": (_cfg(128, 8, 8, 512, "bfloat16"), 24, 1),
    "bf16_long_seq": (_cfg(96, 8, 12, 600, "bfloat16", C=24, D=1640), 3, 40),
}


def _setup(name, seed=13):
    cfg, B, T = CASES[name]
    x = make_inputs(cfg, B, T, seed, variant="rich")
    rng = np.random.default_rng(seed + 1)
    idx = np.stack([rng.choice(cfg.N, cfg.k_max, replace=False) for _ in range(B)]).astype(np.int32)
    a = rng.standard_normal((B, cfg.k_max))
    alphas = (np.exp(a) / np.exp(a).sum(-1, keepdims=True)).astype(np.float32)
    return cfg, x, idx, alphas


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("fused", [False, True])
def test_apply_matches_oracle(name, fused):
    from matrix_b200.assembly import assemble_apply
    from matrix_b200.runtime import raise_on_device_status
    cfg, x, idx, alphas = _setup(name)
    act = torch.bfloat16 if cfg.compute_dtype == "bfloat16" else torch.float32
    pool = _dev(x.pool, torch.bfloat16 if cfg.bf16_pool else torch.float32)
    idx_t = _dev(idx)
    rows = pool if fused else pool[idx_t.long()].contiguous()
    h_mid = assemble_apply(rows, _dev(alphas), _dev(x.h_A, act), _dev(x.W_base), _dev(x.b_base),
                           torch.tensor(x.gamma).cuda(), cfg.d_B, cfg.r, cfg.d_A,
                           row_index=idx_t if fused else None)
    torch.cuda.synchronize()
    raise_on_device_status()
    f = np.float64
    ref_h, _ = O.assemble(x.pool[idx].astype(f), alphas.astype(f), x.h_A.astype(f), x.W_base.astype(f),
                          x.b_base.astype(f), f(x.gamma), cfg.d_B, cfg.r, cfg.d_A)
    tol = BF16_TOL if cfg.compute_dtype == "bfloat16" else F32_TOL
    assert_close(_np(h_mid), ref_h, tol, name="h_mid")


def _torch_factored(pool, idx, alphas, h_A, W_base, b_base, gamma, d, r):
    """Plain PyTorch fp32 statement of the factored apply (assembly_pallas.py:109-117)."""
    B, k = idx.shape
    rows = pool[idx.long()].float()                                   # [B, k, D]
    U = rows[:, :, : d * r].reshape(B, k, d, r)
    V = rows[:, :, d * r: 2 * d * r].reshape(B, k, r, d)
    bv = rows[:, :, 2 * d * r: 2 * d * r + d]
    h = h_A.float()
    hv = torch.einsum("bkri,bti->btkr", V, h) * alphas[:, None, :, None]
    low = torch.einsum("bkjr,btkr->btj", U, hv)
    base = torch.matmul(h, W_base.t())
    pb = b_base[None, :] + torch.einsum("bk,bkj->bj", alphas, bv)
    return h + gamma * (base + low) + pb[:, None, :], h + pb[:, None, :]


@pytest.mark.parametrize("act", ["float32", "bfloat16"])
@pytest.mark.parametrize("B,k,T", [(1, 16, 1), (4, 64, 1), (32, 128, 1), (3, 32, 5)])
def test_apply_matches_torch_fp32_at_decode_shape(B, k, T, act):
    """d 4096, pool rows of 69632 (the decode workload's geometry), against a
    plain PyTorch fp32 statement of the same product (TF32 off).  Float32
    activations: rtol 1e-5 on h_mid - (h_A + pb), i.e. on the two products
    themselves; bfloat16 activations: rtol 2e-2 on h_mid."""
    from matrix_b200.assembly import assemble_apply
    from matrix_b200.runtime import raise_on_device_status
    d, r, N = 4096, 8, 256
    D = d * (2 * r + 1)
    dt = torch.float32 if act == "float32" else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + k + T)
    pool = (torch.randn((N, D), generator=g, device="cuda") * d ** -0.5).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(N, generator=g, device="cuda")[:k] for _ in range(B)]).int()
    alphas = torch.softmax(torch.randn((B, k), generator=g, device="cuda"), -1)
    h_A = torch.randn((B, T, d), generator=g, device="cuda").to(dt)
    W_base = torch.randn((d, d), generator=g, device="cuda") * 0.01
    b_base = torch.randn((d,), generator=g, device="cuda") * 0.1
    gamma = torch.full((1,), 0.5, device="cuda")
    got = assemble_apply(pool, alphas, h_A, W_base, b_base, gamma, d, r, d, row_index=idx)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref, resid = _torch_factored(pool, idx, alphas, h_A, W_base, b_base, gamma, d, r)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    raise_on_device_status()
    if act == "float32":
        assert_close(_np(got - resid), _np(ref - resid).astype(np.float64), F32_TOL, name="products")
    else:
        assert_close(_np(got), _np(ref).astype(np.float64), BF16_TOL, name="h_mid")


def test_apply_bad_row_index_sets_status_bit():
    from matrix_b200.assembly import assemble_apply
    from matrix_b200.runtime import workspace_status
    cfg, x, idx, alphas = _setup("bf16_decode")
    idx = idx.copy()
    idx[2, 5] = cfg.N + 9          # outside the pool: the row contributes nothing, status flags it
    workspace_status(clear=True)
    h_mid = assemble_apply(_dev(x.pool, torch.bfloat16), _dev(alphas), _dev(x.h_A, torch.bfloat16),
                           _dev(x.W_base), _dev(x.b_base), torch.tensor(x.gamma).cuda(),
                           cfg.d_B, cfg.r, cfg.d_A, row_index=_dev(idx))
    st = workspace_status(clear=True)
    assert any(v & 0x1 for v in st.values())      # DWA_STATUS_BAD_ROW_INDEX
    assert torch.isfinite(h_mid.float()).all()
