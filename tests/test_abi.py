"""The C ABI: libdwa.so loads, exports every symbol include/dwa.h declares, and
rejects invalid arguments on the host (no GPU needed: these paths return before
any CUDA call)."""

from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "dwa.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dwa_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from matrix_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from matrix_b200 import build
        build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    from matrix_b200 import _lib
    declared = _declared()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} not exported"
    assert sorted(_lib.exported_symbols()) == declared


def test_version_and_status_strings(lib):
    assert lib.dwa_abi_version() == 1
    assert b"sm_100a" in lib.dwa_version()
    assert lib.dwa_status_string(-1) == b"invalid argument"


def test_invalid_assemble_dims_rejected_on_host(lib):
    from matrix_b200 import _lib
    bad = _lib.AssembleDims(2, 8, 4, 100, 16, 16, 4, 0, 0, 0, 0)   # D < d_B*r + r*d_A + d_B
    assert lib.dwa_assemble_workspace_bytes(bad, 0) == 0
    rc = lib.dwa_assemble_fwd(None, bad, *([None] * 10), None, 0)
    assert rc == -1 and "D < d_B*r" in _lib.last_error()
    uneq = _lib.AssembleDims(2, 8, 4, 4096, 16, 32, 4, 0, 0, 0, 0)  # d_A != d_B
    assert lib.dwa_assemble_fwd(None, uneq, *([None] * 10), None, 0) == -1


def test_workspace_sizes_are_positive_and_aligned(lib):
    from matrix_b200 import _lib
    d = _lib.AssembleDims(8, 512, 32, 17408, 1024, 1024, 8, 1, 1, 0, 262144)
    f = lib.dwa_assemble_workspace_bytes(d, 0)
    b = lib.dwa_assemble_workspace_bytes(d, 1)
    assert f > 0 and b > f and f % 256 == 0
    r = _lib.RetrieveDims(8, 4, 64, 1024, 512, 8, 32, 512, 262144, 1.0, 1)
    assert lib.dwa_retrieve_workspace_bytes(r, 1, 1) > 0
    bad = _lib.RetrieveDims(8, 4, 64, 1024, 512, 8, 300, 512, 262144, 1.0, 1)   # k > 256
    assert lib.dwa_retrieve_workspace_bytes(bad, 1, 1) == 0


def test_missing_workspace_rejected(lib):
    from matrix_b200 import _lib
    d = _lib.AssembleDims(2, 8, 4, 4096, 16, 16, 4, 0, 0, 0, 0)
    p = C.c_void_p(16)
    rc = lib.dwa_assemble_fwd(None, d, p, None, p, p, p, p, p, p, None, None, None, 0)
    assert rc == -4
