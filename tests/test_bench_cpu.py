"""bench.py's host side: the reference arm's restated workload sizes match the
package's workloads, both arms describe a run with the same config, and the
reference arm runs on the host alone (no torch, nothing of matrix_b200
imported)."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)


def test_host_workloads_match_the_package_workloads():
    import bench
    from matrix_b200.config import WORKLOADS
    for name, h in bench.HOST_WORKLOADS.items():
        w = WORKLOADS[name]
        c = w.cfg
        assert (h["B"], h["T"], h["d"], h["N"], h["C"], h["m"], h["k"], h["r"], h["S"], h["dk"]) == \
            (w.batch, w.seq, c.d_A, c.N, c.C, c.m, c.k_max, c.r, c.S, c.d_k), name
        assert (h["zipf"], h["backward"], h["soft_full"], h["lam"], h["warmup"]) == \
            (w.zipf, w.backward, w.soft_full, w.lambda_val, w.is_warmup), name
        assert bench.NOTES[name] == w.note
        assert w.batch % h["sample_B"] == 0


@pytest.mark.parametrize("world", [1, 2, 8])
def test_both_arms_print_the_same_config(world):
    import bench
    from matrix_b200.config import WORKLOADS
    for name in ("medium", "large"):
        ours = bench.run_config(name, world, True, w=WORKLOADS[name])
        ref = bench.run_config(name, world, name in bench.ROWS_WORKLOADS)
        assert ours == ref
        assert ours["parallelism"] == f"rows{world}" and ours["global_batch"] == WORKLOADS[name].batch


SCRIPT = r"""
import json, sys, time
sys.path.insert(0, %r)
import bench
bench.HOST_WORKLOADS["tiny"] = dict(B=4, T=16, d=64, N=4096, C=16, m=4, k=8, r=8, S=4, dk=64, zipf=1.1,
                                    backward=True, soft_full=True, lam=5.0, warmup=False, sample_B=2)
bench.NOTES["tiny"] = "tiny"
x = bench.host_inputs("tiny", 0, n_pool_rows=64)
h = bench.host_step("tiny", x)
assert h.shape == (2, 16, 64) and h.dtype.name == "float32"
class A: workload = "tiny"; seed = 0; steps = 2; warmup = 1; sharded = False
bench.reference_arm(A, 0, 1)
bad = [m for m in sys.modules if m == "torch" or m.startswith("torch.") or m.startswith("matrix_b200")]
print("IMPORTED", json.dumps(bad))
"""


def test_reference_arm_runs_on_the_host_alone():
    out = subprocess.run([sys.executable, "-c", SCRIPT % ROOT], capture_output=True, text=True, timeout=300,
                         env={**os.environ, "OMP_NUM_THREADS": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["cores"] == os.cpu_count()
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert json.loads(lines[-1].split("IMPORTED", 1)[1]) == []
