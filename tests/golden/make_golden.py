"""Generate golden vectors by executing the reference's own hot-path source.

Run in a container that has the reference checkout (read-only is fine)::

    python tests/golden/make_golden.py --reference <reference checkout>

(or set ``DWA_REFERENCE_DIR`` to the checkout instead of passing ``--reference``).

The reference's ``src/dwa/config.py``, ``src/dwa/retrieval.py`` and
``src/dwa/assembly_pallas.py`` are imported unchanged, with JAX / Flax replaced
by the NumPy stand-in in ``numpy_jax.py`` (JAX cannot be installed here).  For
each case the script builds seeded inputs with ``matrix_b200.synthetic``, runs

* ``MultiAspectRetrieval.__call__`` (warmup and gate selection, IVF branch),
* the gather + float32 cast of ``model.py:193-195`` (one line, restated here),
* ``assemble_jax``, ``pallas_assemble`` (Pallas kernel body run per grid step)
  and ``_pallas_assemble_bwd``,

and stores the outputs (float32 / int32) in ``<case>.npz`` next to this file,
together with the SHA-256 of the inputs so a test can confirm it regenerated the
same inputs.  Nothing here runs at test time; the tests only read the ``.npz``.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
sys.path.insert(0, HERE)

from matrix_b200.config import DWAConfig, WORKLOADS  # noqa: E402
from matrix_b200.synthetic import make_inputs  # noqa: E402
import numpy_jax  # noqa: E402

# name -> (config kwargs, batch, seq, seed, variant, modes, with_assembly)
CASES = {
    "smoke": (dict(vars(WORKLOADS["smoke"].cfg)), 2, 128, 0, "spec",
              ((True, 1.0), (False, 5.0)), True),
    "smoke_rich": (dict(vars(WORKLOADS["smoke"].cfg)), 2, 128, 1, "rich",
                   ((True, 1.0), (False, 5.0)), False),
    # the reference's own test dims (config.py:72-80, tests/test_retrieval.py)
    "refsmall": (dict(D=2048, N=512, use_ivf=True, C=128, m=8, d_A=64, d_B=64, r=4, k_max=8,
                      S=2, d_k=32, T=1.0, gamma_init=0.01, bf16_pool=False,
                      compute_dtype="float32"), 4, 64, 2, "rich",
                 ((True, 1.0), (False, 5.0)), True),
    # pad columns (D > s3), B > 8 with B % 8 != 0, odd seq/S/d_k, T != 1
    "ragged": (dict(D=1640, N=6000, use_ivf=True, C=24, m=3, d_A=96, d_B=96, r=8, k_max=12,
                    S=3, d_k=40, T=0.7, gamma_init=0.1, bf16_pool=False,
                    compute_dtype="float32"), 10, 40, 3, "rich",
               ((True, 1.0), (False, 2.5)), True),
}


def run_case(name, ref_config, ref_retrieval, ref_ap):
    kw, B, seq, seed, variant, modes, with_asm = CASES[name]
    cfg = DWAConfig(**kw)
    x = make_inputs(cfg, B, seq, seed, variant=variant)
    rcfg = ref_config.DWAConfig(
        D=cfg.D, N=cfg.N, use_ivf=cfg.use_ivf, C=cfg.C, m=cfg.m, d_A=cfg.d_A, d_B=cfg.d_B,
        r=cfg.r, k_max=cfg.k_max, S=cfg.S, d_k=cfg.d_k, T=cfg.T, n_heads=4, n_kv_heads=1,
        gamma_init=cfg.gamma_init)
    mod = ref_retrieval.MultiAspectRetrieval.__new__(ref_retrieval.MultiAspectRetrieval)
    mod.cfg = rcfg
    mod.W_Q = x.W_Q
    mod.aspect_weights = x.aspect_weights
    mod.tau = np.asarray(x.tau, dtype=np.float32)
    mod.centroids = x.centroids
    out = {"digest": np.array(x.digest()), "B": B, "seq": seq, "seed": seed,
           "variant": np.array(variant)}
    for is_warmup, lam in modes:
        tag = "warmup" if is_warmup else "gate"
        alphas, indices, soft_full = mod(x.z, x.keys, np.float32(lam), is_warmup, mesh=None)
        out[f"{tag}_lambda"] = np.float32(lam)
        out[f"{tag}_alphas"] = np.asarray(alphas, np.float32)
        out[f"{tag}_indices"] = np.asarray(indices, np.int32)
        out[f"{tag}_soft_full"] = np.asarray(soft_full, np.float32)
    if with_asm:
        idx = out["gate_indices"]
        gathered = x.pool[idx].astype(np.float32)          # model.py:193-195
        alphas = out["gate_alphas"]
        gamma = np.asarray(x.gamma, np.float32)
        h_mid, W = ref_ap.assemble_jax(gathered, alphas, x.h_A, x.W_base, x.b_base, gamma,
                                       cfg.d_B, cfg.r, cfg.d_A)
        h_mid_p, W_p = ref_ap.pallas_assemble(gathered, alphas, x.h_A, x.W_base, x.b_base,
                                              gamma, cfg.d_B, cfg.r, cfg.d_A)
        grads = ref_ap._pallas_assemble_bwd(cfg.d_B, cfg.r, cfg.d_A,
                                            (gathered, alphas, x.h_A, W, gamma),
                                            (x.g_hmid, x.g_W))
        out.update(h_mid=h_mid, W=W, h_mid_pallas=h_mid_p, W_pallas=W_p)
        for gname, g in zip(("g_gathered", "g_alpha", "g_hA", "g_W_base", "g_b_base", "g_gamma"),
                            grads):
            out[gname] = np.asarray(g, np.float32)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DWA_REFERENCE_DIR"),
                    help="root of the reference checkout (default: $DWA_REFERENCE_DIR)")
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <checkout> or set DWA_REFERENCE_DIR")
    ref_config, ref_retrieval, ref_ap = numpy_jax.load_reference_modules(
        os.path.join(args.reference, "src", "dwa"))
    for name in args.cases:
        out = run_case(name, ref_config, ref_retrieval, ref_ap)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{name}: {os.path.getsize(path) / 1e3:.0f} kB  digest {str(out['digest'])[:16]}")


if __name__ == "__main__":
    main()
