"""Seeded synthetic inputs for the DWA hot path.

The reference trains on text; the hot path itself only sees a pool, its key
cache, IVF centroids/lists, activations and the retrieval parameters.  These
are generated here with ``numpy.random.default_rng(seed)`` using the
reference's initialisation scales where it has them:

* pool rows ``~ N(0, 1/sqrt(d))`` (the workload spec; the reference's own init
  is ``0.02``, src/dwa/pool.py:29)
* key projection ``~ N(0, 1/sqrt(D))`` (pool.py:32-35), keys = ``pool @ key_proj``
  in float32 (pool.py:37-44, assembly_pallas.py:392-400)
* ``W_Q ~ N(0, 1/sqrt(d_A))`` (retrieval.py:36-38)
* ``W_base ~ 0.01 N(0,1)`` (assembly.py:24-26), ``gamma = cfg.gamma_init``
* centroid ``c`` = the key of a random row of list ``c``
* ``h_A ~ N(0,1)``, ``z = mean_t h_A`` (model.py:171)

``variant="rich"`` additionally randomises ``aspect_weights``, ``tau`` and
``b_base`` (all zero at reference init) so that tests exercise those terms.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

from .config import DWAConfig


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit pattern (uint16), round to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def zipf_list_offsets(N: int, C: int, s: float, rng: np.random.Generator) -> np.ndarray:
    """CSR offsets for ``C`` lists whose sizes follow Zipf(s), summing to ``N``,
    every list non-empty, in a random order."""
    w = 1.0 / np.arange(1, C + 1, dtype=np.float64) ** s
    sizes = np.floor(w / w.sum() * (N - C)).astype(np.int64) + 1
    sizes[0] += N - sizes.sum()
    rng.shuffle(sizes)
    off = np.zeros(C + 1, dtype=np.int64)
    np.cumsum(sizes, out=off[1:])
    return off


@dataclass
class HotPathInputs:
    """All inputs of one retrieval + assembly step, as NumPy arrays.

    Float arrays hold exactly representable values of the workload dtype
    (bf16-rounded when the workload is bf16), stored as float32.
    """

    pool: np.ndarray          # [N, D]
    keys: np.ndarray          # [S, N, d_k] float32
    list_offsets: np.ndarray  # [C+1] int64
    centroids: np.ndarray     # [S, C, d_k]
    W_Q: np.ndarray           # [S, d_k, d_A]
    aspect_weights: np.ndarray  # [S]
    tau: float
    W_base: np.ndarray        # [d_B, d_A]
    b_base: np.ndarray        # [d_B]
    gamma: float
    h_A: np.ndarray           # [B, seq, d_A]
    z: np.ndarray             # [B, d_A] float32
    g_hmid: np.ndarray        # [B, seq, d_B]
    g_W: np.ndarray           # [B, d_B, d_A]
    key_proj: np.ndarray | None = None   # [S, D, d_k], keys = pool @ key_proj (not in the digest)

    def digest(self) -> str:
        h = hashlib.sha256()
        for name in ("pool", "keys", "list_offsets", "centroids", "W_Q", "aspect_weights",
                     "W_base", "b_base", "h_A", "g_hmid", "g_W"):
            h.update(np.ascontiguousarray(getattr(self, name)).tobytes())
        h.update(np.float64(self.tau).tobytes())
        h.update(np.float64(self.gamma).tobytes())
        return h.hexdigest()


def make_inputs(cfg: DWAConfig, batch: int, seq: int, seed: int = 0, *,
                variant: str = "spec", zipf: float | None = None,
                pool_rows: np.ndarray | None = None) -> HotPathInputs:
    """Generate one seeded input set on the host.

    ``pool_rows``, if given, replaces the generated pool (used to share one pool
    between several parity cases).
    """
    rng = np.random.default_rng(seed)
    d, D, N, S, dk = cfg.d_A, cfg.D, cfg.N, cfg.S, cfg.d_k
    bf16 = cfg.compute_dtype == "bfloat16"
    pool_bf16 = cfg.bf16_pool
    f32 = np.float32

    if pool_rows is None:
        pool = rng.standard_normal((N, D), dtype=f32) * f32(1.0 / np.sqrt(d))
    else:
        pool = np.asarray(pool_rows, dtype=f32)
        rng.standard_normal(1)
    key_proj = rng.standard_normal((S, D, dk), dtype=f32) * f32(1.0 / np.sqrt(D))
    if pool_bf16:
        pool = bf16_round(pool)
        key_proj = bf16_round(key_proj)
    keys = np.einsum("nd,sda->sna", pool, key_proj).astype(f32)

    if zipf is None:
        if N % cfg.C != 0:
            raise ValueError("equal lists need N % C == 0")
        offsets = (np.arange(cfg.C + 1, dtype=np.int64) * (N // cfg.C))
    else:
        offsets = zipf_list_offsets(N, cfg.C, zipf, rng)
    rows = np.array([rng.integers(offsets[c], offsets[c + 1]) for c in range(cfg.C)])
    centroids = np.ascontiguousarray(keys[:, rows, :])

    W_Q = rng.standard_normal((S, dk, d), dtype=f32) * f32(d ** -0.5)
    if variant == "rich":
        aspect_weights = rng.standard_normal(S, dtype=f32) * f32(0.5)
        tau = float(np.float32(0.05))
        b_base = rng.standard_normal(cfg.d_B, dtype=f32) * f32(0.01)
    else:
        aspect_weights = np.zeros(S, dtype=f32)
        tau = 0.0
        b_base = np.zeros(cfg.d_B, dtype=f32)
    W_base = rng.standard_normal((cfg.d_B, d), dtype=f32) * f32(0.01)
    gamma = float(np.float32(cfg.gamma_init))

    h_A = rng.standard_normal((batch, seq, d), dtype=f32)
    g_hmid = rng.standard_normal((batch, seq, cfg.d_B), dtype=f32) * f32(0.1)
    g_W = rng.standard_normal((batch, cfg.d_B, d), dtype=f32) * f32(0.001)
    if bf16:
        h_A = bf16_round(h_A)
        g_hmid = bf16_round(g_hmid)
    z = h_A.mean(axis=1, dtype=np.float64).astype(f32)
    return HotPathInputs(pool=pool, keys=keys, list_offsets=offsets.astype(np.int64),
                         centroids=centroids, W_Q=W_Q, aspect_weights=aspect_weights,
                         tau=tau, W_base=W_base, b_base=b_base, gamma=gamma, h_A=h_A, z=z,
                         g_hmid=g_hmid, g_W=g_W, key_proj=key_proj)
