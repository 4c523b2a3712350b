"""``sequence_mean`` (``dwa_sequence_mean``, z = h_A.mean(axis=1) at
model.py:171) against numpy in float64, rtol 1e-5: bf16 and f32 inputs, row
counts that split the sum over 1, 3 and 8 CTAs of a cluster, a width that is
not a multiple of 8 (the 2-column kernel), and bit-identical repeats."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.synthetic import bf16_round

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,d,bf16", [
    (8, 512, 1024, True),     # 8 CTAs per cluster
    (3, 150, 96, False),      # 3 CTAs per cluster, one column block partly used
    (2, 40, 2048, True),      # one CTA
    (4, 2048, 264, False),    # 8 CTAs, 256 rows each
    (2, 37, 100, False),      # d % 8 != 0
])
def test_sequence_mean_matches_numpy(B, T, d, bf16):
    from matrix_b200.retrieval import sequence_mean
    rng = np.random.default_rng(B * T + d)
    h = rng.standard_normal((B, T, d), dtype=np.float32)
    if bf16:
        h = bf16_round(h)
    dt = torch.bfloat16 if bf16 else torch.float32
    hd = torch.from_numpy(h).cuda().to(dt)
    z = sequence_mean(hd)
    ref = h.astype(np.float64).mean(axis=1)
    assert_close(z.cpu().numpy(), ref, 1e-5, name=f"z B={B} T={T} d={d}")
    np.testing.assert_array_equal(sequence_mean(hd).cpu().numpy(), z.cpu().numpy())
