"""Selection paths of the CUDA retrieval at list counts, probe counts and top-k
sizes the golden-vector cases do not reach, against the oracle in float64:

* 512 lists, nprobe 8, top-k 32, four aspects (the single-GPU workload's
  retrieval shape on a smaller pool): one cluster of 8 CTAs per query scores
  the lists and picks the probes;
* one aspect (64 threads per CTA) with nprobe 100 of 200 lists: the top-m
  sort has fewer threads than slots; top-k 64: the final sort exchanges
  through shared memory once;
* 6200 lists: more list keys than shared memory holds, so normalisation,
  coarse scores and top-m run as three kernels; top-k 128;
* 15 probes of 8000-row lists: 120000 candidates, more than a cluster
  stages at once, so each CTA takes its share in two passes and carries its
  running winners from the first into the second.

Each case runs with and without soft_full (selection from the full pass and
from the fine pass).  Indices equal the oracle's (seed 40 leaves a gap above
1e-5 at the list and top-k boundaries of every query, checked here too);
alphas and soft_full within rtol 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs
from oracle import dwa_oracle as O
from test_gpu_retrieval import TOL, _gpu_retrieve

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("C,m,k,S,list_len,B", [
    (512, 8, 32, 4, 40, 8),
    (200, 100, 64, 1, 20, 3),
    (6200, 16, 128, 1, 10, 13),
    (20, 15, 48, 1, 8000, 3),
])
@pytest.mark.parametrize("is_warmup,lam", [(True, 1.0), (False, 5.0)])
def test_selection_paths_match_oracle(C, m, k, S, list_len, B, is_warmup, lam):
    from matrix_b200.runtime import raise_on_device_status
    cfg = DWAConfig(D=17 * 64, N=C * list_len, use_ivf=True, C=C, m=m, d_A=64, d_B=64, r=8, k_max=k,
                    S=S, d_k=64, T=1.0, gamma_init=0.1, bf16_pool=False)
    x = make_inputs(cfg, B, 8, 40, variant="rich")
    f = np.float64
    ra, ri, rsf, it = O.retrieve(x.z.astype(f), x.W_Q.astype(f), x.aspect_weights.astype(f), f(x.tau),
                                 x.centroids.astype(f), x.keys.astype(f), k=k, m=m, T=cfg.T,
                                 lambda_val=lam, is_warmup=is_warmup, list_offsets=x.list_offsets,
                                 tie_break="index", return_internals=True)
    c = np.sort(it["c_score"], axis=1)[:, ::-1]
    assert (c[:, m - 1] - c[:, m] > 1e-5).all(), "seed has a near-tie among lists"
    for b in range(B):
        s = np.sort(it["s_i"][b])[::-1]
        assert s[k - 1] - s[k] > 1e-5, "seed has a near-tie at top-k"
    tag = f"C={C} m={m} k={k} S={S} warmup={is_warmup}"
    a, i, sf = _gpu_retrieve(cfg, x, lam, is_warmup, True)
    np.testing.assert_array_equal(i, ri, err_msg=tag)
    assert_close(a, ra, TOL, name=f"alphas {tag}")
    assert_close(sf, rsf, TOL, name=f"soft_full {tag}")
    a2, i2, _ = _gpu_retrieve(cfg, x, lam, is_warmup, False)
    np.testing.assert_array_equal(i2, i, err_msg=f"fine pass {tag}")
    np.testing.assert_array_equal(a2, a, err_msg=f"fine pass {tag}")
    raise_on_device_status()
