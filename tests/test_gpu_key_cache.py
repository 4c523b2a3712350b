"""Key cache (``dwa_key_cache``) and centroid EMA (``dwa_centroid_ema``) on the GPU.

* keys = einsum("nd,sda->sna", pool, key_proj) (assembly_pallas.py:392-400)
  against the oracle in float64, rtol 1e-5: bf16 inputs on the tensor-core
  GEMM with 256- and 128-column tiles (the second with a row tail and a
  K tail), bf16 on the CUDA-core GEMM (S * d_k < 128), f32 on the CUDA-core GEMM.
* The reference's key-cache test (tests/test_model.py:88-93) in retrieval
  terms: retrieval on the computed keys selects what it selects on the
  oracle's keys.
* Centroid EMA (train.py:318-328) on equal lists and on Zipf lists with an
  empty list, against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.synthetic import bf16_round
from oracle import dwa_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def _inputs(N, D, S, d_k, bf16, seed):
    rng = np.random.default_rng(seed)
    pool = rng.standard_normal((N, D), dtype=np.float32) * np.float32(D ** -0.5)
    kp = rng.standard_normal((S, D, d_k), dtype=np.float32) * np.float32(D ** -0.5)
    if bf16:
        pool, kp = bf16_round(pool), bf16_round(kp)
    return pool, kp


@pytest.mark.parametrize("N,D,S,d_k,bf16", [
    (20480, 1088, 4, 64, True),    # 160 row tiles: 256-column tensor-core tiles
    (6181, 680, 4, 64, True),      # 49 row tiles, rows and K not tile multiples: 128-column tiles
    (3000, 544, 2, 32, True),      # S * d_k = 64: CUDA-core GEMM on bf16
    (3001, 300, 4, 64, False),     # f32: CUDA-core GEMM
])
def test_key_cache_matches_oracle(N, D, S, d_k, bf16):
    from matrix_b200.assembly import compute_key_cache
    from matrix_b200.runtime import raise_on_device_status
    pool, kp = _inputs(N, D, S, d_k, bf16, seed=N + D)
    dt = torch.bfloat16 if bf16 else torch.float32
    keys = compute_key_cache(torch.from_numpy(pool).cuda().to(dt), torch.from_numpy(kp).cuda().to(dt))
    torch.cuda.synchronize()
    ref = O.compute_key_cache(pool.astype(np.float64), kp.astype(np.float64))
    assert keys.shape == (S, N, d_k) and keys.dtype == torch.float32
    assert_close(keys.cpu().numpy(), ref, TOL, name=f"keys N={N} D={D} S={S} d_k={d_k} bf16={bf16}")
    raise_on_device_status()


def test_retrieval_on_computed_keys_matches_oracle_keys():
    """tests/test_model.py:88-93 (cached vs recomputed keys give the same model
    output) as a retrieval check: same indices, alphas within 1e-5."""
    from matrix_b200.assembly import compute_key_cache
    from matrix_b200.config import DWAConfig
    from matrix_b200.retrieval import retrieve
    from matrix_b200.synthetic import make_inputs
    cfg = DWAConfig(D=17 * 64, N=20480, use_ivf=True, C=40, m=5, d_A=64, d_B=64, r=8, k_max=24,
                    S=4, d_k=64, T=1.0, gamma_init=0.1, bf16_pool=True)
    x = make_inputs(cfg, 4, 8, 8, variant="rich")
    keys = compute_key_cache(torch.from_numpy(x.pool).cuda().bfloat16(),
                             torch.from_numpy(x.key_proj).cuda().bfloat16())

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    outs = []
    for kc in (keys, d(x.keys)):
        a, i, _ = retrieve(d(x.z), d(x.W_Q), d(x.aspect_weights), torch.tensor(x.tau).cuda(),
                           d(x.centroids), kc, 5.0, False, k=cfg.k_max, m=cfg.m, T=cfg.T,
                           want_soft_full=False)
        outs.append((a.cpu().numpy(), i.cpu().numpy()))
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    assert_close(outs[0][0], outs[1][0], TOL, name="alphas")


@pytest.mark.parametrize("zipf", [False, True])
def test_centroid_ema_matches_oracle(zipf):
    from matrix_b200.assembly import centroid_ema
    from matrix_b200.synthetic import zipf_list_offsets
    rng = np.random.default_rng(5)
    S, N, C, d_k = 4, 12000, 48, 64
    keys = rng.standard_normal((S, N, d_k), dtype=np.float32)
    cent = rng.standard_normal((S, C, d_k), dtype=np.float32)
    if zipf:
        off = zipf_list_offsets(N, C, 1.1, rng).astype(np.int64)
        off[7] = off[8] = (off[6] + off[9]) // 2     # list 7 is empty, list 8 takes its rows
        off = np.maximum.accumulate(off)
    else:
        off = np.arange(C + 1, dtype=np.int64) * (N // C)
    c_dev = torch.from_numpy(cent.copy()).cuda()
    centroid_ema(c_dev, torch.from_numpy(keys).cuda(), torch.from_numpy(off).cuda(), 0.9)
    torch.cuda.synchronize()
    ref = O.centroid_ema(cent.astype(np.float64), keys.astype(np.float64), off, 0.9)
    assert_close(c_dev.cpu().numpy(), ref, TOL, name=f"centroids zipf={zipf}")
    if zipf:
        np.testing.assert_array_equal(c_dev.cpu().numpy()[:, 7], cent[:, 7])
