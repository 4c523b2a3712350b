"""Hot-path configuration: the DWA config keys the retrieval and assembly use.

``DWAConfig`` keeps the reference's field names, defaults and asserts for the
keys the hot path consumes (src/dwa/config.py:7-70, ``factor_split`` :159-165).
Transformer, trainer and loader keys are not part of this path and are not
carried.

``WORKLOADS`` names the synthetic workloads the parity tests and the benchmark
run.  Pool rows follow the reference's ``[U | V | b]`` layout, so the pool row
width is ``D = d*(2r+1)`` with ``r = 8`` and ``d_A = d_B = d``; ``S = 4``,
``d_k = 64`` and the temperature ``T = 1.0`` are the reference defaults.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass
class DWAConfig:
    """Hot-path subset of the reference ``DWAConfig`` (src/dwa/config.py:7-165)."""

    D: int = 16384          # pool vector dim
    N: int = 65536          # pool size
    use_ivf: bool = True    # two-stage IVF retrieval
    C: int = 128            # number of lists (centroids)
    m: int = 8              # lists probed per query
    d_A: int = 256
    d_B: int = 256
    r: int = 24             # low-rank factors per pool vector
    k_max: int = 16         # vectors retrieved per query
    S: int = 4              # retrieval aspects
    d_k: int = 64           # key/query dim per aspect
    T: float = 1.0          # temperature
    gamma_init: float = 0.01
    bf16_pool: bool = True
    compute_dtype: str = "float32"   # activation dtype: "float32" or "bfloat16"

    def __post_init__(self):
        # Same checks as the reference (config.py:53-70).
        needed = self.d_B * self.r + self.r * self.d_A + self.d_B
        if self.D < needed:
            raise ValueError(f"D={self.D} < needed={needed} (d_B*r + r*d_A + d_B)")
        if self.d_A != self.d_B:
            raise ValueError("d_A must equal d_B for the residual connection")
        if self.use_ivf:
            if self.N % self.C != 0:
                raise ValueError(f"N={self.N} must be divisible by C={self.C} for IVF equal-size buckets")
            if self.m > self.C:
                raise ValueError(f"m={self.m} (clusters searched) must be <= C={self.C}")

    @property
    def factor_split(self) -> tuple[int, int, int]:
        """``(s1, s2, s3)`` offsets of U, V, b inside a pool row (config.py:159-165)."""
        s1 = self.d_B * self.r
        s2 = s1 + self.r * self.d_A
        return s1, s2, s2 + self.d_B

    @classmethod
    def small(cls) -> "DWAConfig":
        """The reference's test config (config.py:72-80), hot-path keys only."""
        return cls(D=2048, N=512, d_A=64, d_B=64, r=4, k_max=8, S=2, d_k=32)


@dataclass(frozen=True)
class Workload:
    """A named synthetic workload: a config plus batch and sequence length."""

    name: str
    cfg: DWAConfig
    batch: int
    seq: int
    backward: bool
    lambda_val: float = 5.0
    is_warmup: bool = False
    soft_full: bool = True
    zipf: float | None = None   # Zipf exponent of the list sizes (None: equal lists)
    note: str = ""


def _cfg(d, N, C, m, k, dtype, r=8):
    return DWAConfig(D=d * (2 * r + 1), N=N, use_ivf=True, C=C, m=m, d_A=d, d_B=d, r=r,
                     k_max=k, S=4, d_k=64, T=1.0, gamma_init=0.1,
                     bf16_pool=(dtype == "bfloat16"), compute_dtype=dtype)


WORKLOADS: dict[str, Workload] = {
    "smoke": Workload("smoke", _cfg(256, 8192, 64, 4, 16, "float32"), 2, 128, True,
                      note="fp32, batch 2, seq 128, d 256, pool 8192, 64 lists, nprobe 4, top-k 16"),
    "small": Workload("small", _cfg(1024, 262144, 512, 8, 32, "bfloat16"), 8, 512, True,
                      note="bf16, batch 8, seq 512, d 1024, pool 262144, 512 lists, nprobe 8, top-k 32, fwd+bwd"),
    "medium": Workload("medium", _cfg(2048, 1 << 20, 1024, 16, 64, "bfloat16"), 16, 1024, False,
                       note="bf16, batch 16, seq 1024, d 2048, pool 1M, 1024 lists, nprobe 16, top-k 64, fwd"),
    "large": Workload("large", _cfg(2048, 1 << 22, 4096, 32, 64, "bfloat16"), 32, 2048, True,
                      zipf=1.1,
                      note="bf16, batch 32, seq 2048, d 2048, pool 4M, 4096 Zipf(1.1) lists, nprobe 32, top-k 64"),
    "decode": Workload("decode", _cfg(4096, 1 << 21, 2048, 16, 64, "bfloat16"), 64, 1, False,
                       note="bf16, batch 1-256, seq 1, d 4096, pool 2M, 2048 lists, nprobe 16, top-k 16-128"),
    # reduced cases for detailed ncu captures (a few GB on the device)
    "decode_profile": Workload("decode_profile", _cfg(4096, 1 << 14, 16, 16, 128, "bfloat16"), 256, 1, False,
                               note="ncu case: decode shapes (d 4096, batch 256, top-k 128) on a 2.3 GB pool "
                                    "of 16384 rows in 16 lists"),
    "profile_keys": Workload("profile_keys", _cfg(512, 131072, 256, 8, 32, "bfloat16"), 8, 512, True,
                             note="ncu case: key cache 134 MB (> L2), pool 2.3 GB; small shapes otherwise"),
    "profile_scan16": Workload("profile_scan16", _cfg(512, 131072, 256, 8, 32, "bfloat16"), 16, 256, False,
                               note="ncu case: the 16-query key scan over a 134 MB key cache (> L2), forward"),
    "profile_gemm2k": Workload("profile_gemm2k", _cfg(2048, 16384, 16, 8, 64, "bfloat16"), 8, 1024, False,
                               note="ncu case: the medium workload's assembly GEMM shapes (d 2048, top-k 64, "
                                    "seq 1024) for 8 sequences on a 1.1 GB pool (the W GEMM's grid is multi-wave "
                                    "enough for the persistent kernel, as on the medium batch)"),
    "profile_gemm": Workload("profile_gemm", _cfg(1024, 16384, 32, 8, 32, "bfloat16"), 8, 512, True,
                             note="ncu case: the small workload's GEMM shapes with a 0.57 GB pool"),
}


def scaled(w: Workload, **changes) -> Workload:
    """A copy of ``w`` with config fields and/or batch/seq replaced."""
    wfields = {k: changes.pop(k) for k in list(changes) if k in ("batch", "seq", "backward",
                                                                   "lambda_val", "is_warmup",
                                                                   "soft_full", "zipf", "name")}
    cfg = replace(w.cfg, **changes) if changes else w.cfg
    return replace(w, cfg=cfg, **wfields)
