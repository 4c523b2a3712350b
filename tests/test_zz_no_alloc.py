"""dwa_retrieve_noalloc: retrieval for callers that cannot pass a workspace or
let the library allocate (for example a legacy XLA custom-call target, which
only receives its operand and result buffers, or code running under CUDA stream
capture, where cudaMalloc is not allowed).  It uses a fixed 8 MiB scratch array
inside libdwa instead of a workspace.

The GPU test calls it through the C ABI twice in a row and checks each result
against the workspace entry point dwa_retrieve on the same inputs: indices
identical, alphas and soft_full within the retrieval tolerance (rtol 1e-5).
It then reads the device status word back through dwa_retrieve_noalloc_status:
clear after the good calls, the list-overflow bit after a call whose max_list
is shorter than the probed lists (the kernels clip such a list and flag it),
and clear again after the next good call, since every call starts from zero.
This file is collected last so a run that stops at the first failure has run
every other test before it.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from matrix_b200.config import DWAConfig
from matrix_b200.synthetic import make_inputs

TOL = 1e-5


def _case():
    cfg = DWAConfig(D=17 * 64, N=6144, use_ivf=True, C=48, m=4, d_A=64, d_B=64, r=8, k_max=16,
                    S=4, d_k=64, T=1.0, gamma_init=0.1, bf16_pool=False)
    return cfg, make_inputs(cfg, 3, 8, 31, variant="rich")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from matrix_b200 import _lib
    lib = _lib.load()
    # full search without soft_full needs B*N*4 bytes of raw scores: 64 * 262144 * 4 > 8 MiB
    big = _lib.RetrieveDims(64, 4, 64, 1024, 1, 1, 32, 1, 262144, 1.0, 0)
    rc = lib.dwa_retrieve_noalloc(None, big, 0, 1, *([None] * 11))
    assert rc == -2
    assert "built-in scratch" in _lib.last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls():
    torch = pytest.importorskip("torch")
    from matrix_b200 import _lib
    from matrix_b200.runtime import ptr, stream_of
    lib = _lib.load()
    cfg, x = _case()
    dev = torch.device("cuda", 0)

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    z, W_Q, aw = d(x.z), d(x.W_Q), d(x.aspect_weights)
    tau, cents, keys = d(np.array([x.tau], np.float32)), d(x.centroids), d(x.keys)
    off = d(x.list_offsets)
    B, N, k = z.shape[0], cfg.N, cfg.k_max
    dims = _lib.RetrieveDims(B, cfg.S, cfg.d_k, cfg.d_A, cfg.C, cfg.m, k, N // cfg.C, N, cfg.T,
                             _lib.DWA_F32)
    st = stream_of(dev)
    for is_warmup, lam_v in ((True, 1.0), (False, 5.0)):
        lam = d(np.array([lam_v], np.float32))
        for want_sf in (True, False):
            nbytes = lib.dwa_retrieve_workspace_bytes(dims, 1, int(want_sf))
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            for call in range(2):
                outs = []
                for noalloc in (False, True):
                    a = torch.full((B, k), -1.0, device=dev)
                    i = torch.full((B, k), -1, dtype=torch.int32, device=dev)
                    sf = torch.full((B, N), -1.0, device=dev) if want_sf else None
                    args = (st, dims, 1, int(is_warmup), ptr(lam), ptr(z), ptr(W_Q), ptr(aw),
                            ptr(tau), ptr(cents), ptr(off), ptr(keys), ptr(a), ptr(i), ptr(sf))
                    if noalloc:
                        rc = lib.dwa_retrieve_noalloc(*args)
                    else:
                        rc = lib.dwa_retrieve(*args, ptr(ws), C.c_size_t(nbytes))
                    _lib.check(rc, "noalloc" if noalloc else "workspace")
                    torch.cuda.synchronize()
                    outs.append((a.cpu().numpy(), i.cpu().numpy(),
                                 None if sf is None else sf.cpu().numpy()))
                (a1, i1, s1), (a2, i2, s2) = outs
                tag = f"warmup={is_warmup} soft_full={want_sf} call={call}"
                np.testing.assert_array_equal(i2, i1, err_msg=tag)
                assert_close(a2, a1, TOL, name=f"alphas {tag}")
                if want_sf:
                    assert_close(s2, s1, TOL, name=f"soft_full {tag}")

    # the status word: clean after the good calls above
    bits = C.c_uint32(0xFFFFFFFF)
    assert lib.dwa_retrieve_noalloc_status(st, C.byref(bits), 1) == 0
    assert bits.value == 0
    # a max_list shorter than the lists (128 rows each): clipped and flagged
    short = _lib.RetrieveDims(B, cfg.S, cfg.d_k, cfg.d_A, cfg.C, cfg.m, k, 64, N, cfg.T, _lib.DWA_F32)
    a = torch.empty((B, k), device=dev)
    i = torch.empty((B, k), dtype=torch.int32, device=dev)
    lam = d(np.array([5.0], np.float32))
    for dims_, expect in ((short, 0x8), (dims, 0)):
        _lib.check(lib.dwa_retrieve_noalloc(st, dims_, 1, 0, ptr(lam), ptr(z), ptr(W_Q), ptr(aw), ptr(tau),
                                            ptr(cents), ptr(off), ptr(keys), ptr(a), ptr(i), None),
                   "noalloc")
        rc = lib.dwa_retrieve_noalloc_status(st, C.byref(bits), 0)
        assert bits.value == expect, (bits.value, expect)
        assert rc == (0 if expect == 0 else _lib.DWA_ERR_DEVICE)
