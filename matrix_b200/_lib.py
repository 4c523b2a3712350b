"""ctypes binding of libdwa.so (the C ABI declared in include/dwa.h).

The library is built in-tree (``matrix_b200/libdwa.so``, see ``build.py``).
Loading fails loudly when it is missing: the hot path has no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdwa.so")

DWA_OK = 0
DWA_ERR_DEVICE = -5
DWA_PAD_INDEX = -(2 ** 31)
DWA_F32 = 0
DWA_BF16 = 1

STATUS_BITS = {
    0x1: "row index outside the pool",
    0x2: "a bounded device wait ran out",
    0x4: "list offsets not monotone or out of range",
    0x8: "a probed list is longer than max_list",
    0x10: "fewer candidates than k",
}


class DwaError(RuntimeError):
    """An error returned by libdwa (the message is the library's last error)."""


class AssembleDims(C.Structure):
    _fields_ = [("B", C.c_int32), ("T", C.c_int32), ("k", C.c_int32), ("D", C.c_int32),
                ("d_A", C.c_int32), ("d_B", C.c_int32), ("r", C.c_int32),
                ("act_dtype", C.c_int32), ("rows_dtype", C.c_int32), ("reserved", C.c_int32),
                ("n_rows", C.c_int64)]


class RetrieveDims(C.Structure):
    _fields_ = [("B", C.c_int32), ("S", C.c_int32), ("d_k", C.c_int32), ("d_A", C.c_int32),
                ("C", C.c_int32), ("m", C.c_int32), ("k", C.c_int32), ("max_list", C.c_int32),
                ("N", C.c_int64), ("T", C.c_float), ("z_dtype", C.c_int32)]


class KeyCacheDims(C.Structure):
    _fields_ = [("N", C.c_int64), ("D", C.c_int32), ("S", C.c_int32), ("d_k", C.c_int32),
                ("dtype", C.c_int32)]


class Shard(C.Structure):
    _fields_ = [("row_lo", C.c_int64), ("n_global", C.c_int64)]


class PoolShards(C.Structure):
    _fields_ = [("world", C.c_int32), ("bases", C.POINTER(C.c_void_p)), ("row_lo", C.POINTER(C.c_int64))]


class AuxDims(C.Structure):
    _fields_ = [("B", C.c_int32), ("k", C.c_int32), ("S", C.c_int32), ("d_k", C.c_int32),
                ("d_B", C.c_int32), ("d_A", C.c_int32), ("N", C.c_int64)]


class AuxShard(C.Structure):
    _fields_ = [("row_lo", C.c_int64), ("n_global", C.c_int64), ("w_batch", C.c_int32)]


class AuxWeights(C.Structure):
    _fields_ = [("util", C.c_float), ("div", C.c_float), ("norm", C.c_float), ("sparse", C.c_float)]


_P = C.c_void_p
_SIGNATURES = {
    "dwa_version": (C.c_char_p, []),
    "dwa_abi_version": (C.c_int, []),
    "dwa_status_string": (C.c_char_p, [C.c_int]),
    "dwa_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "dwa_workspace_status": (C.c_int, [_P, _P, C.POINTER(C.c_uint32), C.c_int]),
    "dwa_launch_counters": (None, [C.POINTER(C.c_uint64)] * 3),
    "dwa_profile_kernel": (C.c_int, [C.c_char_p, _P, _P]),
    "dwa_profile_clear": (None, []),
    "dwa_profile_serialize": (None, [C.c_int]),
    "dwa_sequence_mean": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P]),
    "dwa_assemble_workspace_bytes": (C.c_size_t, [C.POINTER(AssembleDims), C.c_int]),
    "dwa_assemble_fwd": (C.c_int, [_P, C.POINTER(AssembleDims), _P, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _P, _P, C.c_size_t]),
    "dwa_assemble_apply_workspace_bytes": (C.c_size_t, [C.POINTER(AssembleDims)]),
    "dwa_assemble_apply": (C.c_int, [_P, C.POINTER(AssembleDims), _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                     C.c_size_t]),
    "dwa_assemble_bwd": (C.c_int, [_P, C.POINTER(AssembleDims), _P, _P, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_workspace_bytes": (C.c_size_t, [C.POINTER(RetrieveDims), C.c_int, C.c_int]),
    "dwa_retrieve": (C.c_int, [_P, C.POINTER(RetrieveDims), C.c_int, C.c_int, _P, _P, _P, _P, _P,
                               _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_noalloc": (C.c_int, [_P, C.POINTER(RetrieveDims), C.c_int, C.c_int, _P, _P, _P,
                                       _P, _P, _P, _P, _P, _P, _P, _P]),
    "dwa_retrieve_noalloc_status": (C.c_int, [_P, C.POINTER(C.c_uint32), C.c_int]),
    "dwa_retrieve_local": (C.c_int, [_P, C.POINTER(RetrieveDims), C.POINTER(Shard), C.c_int, C.c_int,
                                     _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_merge_workspace_bytes": (C.c_size_t, [C.POINTER(RetrieveDims)]),
    "dwa_key_cache_workspace_bytes": (C.c_size_t, [C.POINTER(KeyCacheDims)]),
    "dwa_rmsnorm_fwd": (C.c_int, [_P, C.c_int64, C.c_int, C.c_int, C.c_int, _P, _P, C.c_float, _P, _P]),
    "dwa_rmsnorm_bwd_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int]),
    "dwa_pool_grad_scatter_workspace_bytes": (C.c_size_t, [C.c_int]),
    "dwa_pool_grad_scatter": (C.c_int, [_P, C.c_int, C.c_int, _P, _P, C.c_int64, C.c_int64, C.c_int64,
                                        C.c_int, _P, _P, C.c_size_t]),
    "dwa_pool_grad_scatter_typed": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_int64, C.c_int64,
                                              C.c_int64, C.c_int, _P, _P, C.c_size_t]),
    "dwa_pool_grad_recv_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int64, C.c_int]),
    "dwa_pool_grad_send": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int64, _P, _P, C.c_int,
                                     C.POINTER(PoolShards), _P, C.c_size_t]),
    "dwa_peer_allgather_buffer_bytes": (C.c_size_t, [C.c_int, C.c_size_t]),
    "dwa_peer_allgather": (C.c_int, [_P, C.c_int, C.c_int, _P, C.c_size_t, C.POINTER(_P), _P]),
    "dwa_peer_allgather_status": (C.c_int, [_P, _P, C.POINTER(C.c_uint32), C.c_int]),
    "dwa_rmsnorm_bwd": (C.c_int, [_P, C.c_int64, C.c_int, C.c_int, C.c_int, _P, _P, _P, _P, _P, _P, _P,
                                  C.c_size_t]),
    "dwa_key_cache": (C.c_int, [_P, C.POINTER(KeyCacheDims), _P, _P, _P, _P, C.c_size_t]),
    "dwa_centroid_ema": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int64, _P, _P, C.c_float, _P, _P,
                                   C.c_size_t]),
    "dwa_retrieve_bwd_local_workspace_bytes": (C.c_size_t, [C.POINTER(RetrieveDims), C.c_int]),
    "dwa_retrieve_bwd_local1": (C.c_int, [_P, C.POINTER(RetrieveDims), C.POINTER(Shard), C.c_int, C.c_int,
                                          _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_bwd_local2": (C.c_int, [_P, C.POINTER(RetrieveDims), C.POINTER(Shard), C.c_int, C.c_int,
                                          _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_bwd_finish": (C.c_int, [_P, C.POINTER(RetrieveDims), C.c_int, _P, _P, _P, _P, _P, _P, _P, _P,
                                          _P, C.c_size_t]),
    "dwa_ipc_handle_bytes": (C.c_size_t, []),
    "dwa_ipc_handle": (C.c_int, [_P, _P, C.POINTER(C.c_int64)]),
    "dwa_ipc_open": (C.c_int, [_P, C.c_int64, C.POINTER(C.c_void_p)]),
    "dwa_ipc_close": (C.c_int, [_P, C.c_int64]),
    "dwa_gather_rows_workspace_bytes": (C.c_size_t, []),
    "dwa_gather_rows": (C.c_int, [_P, C.c_int, C.c_int64, C.c_int, _P, C.POINTER(PoolShards), _P, _P, C.c_size_t]),
    "dwa_aux_losses_local": (C.c_int, [_P, C.POINTER(AuxDims), C.POINTER(AuxShard), C.POINTER(AuxWeights),
                                       _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_aux_losses_finish": (C.c_int, [_P, C.POINTER(AuxDims), C.POINTER(AuxShard), C.POINTER(AuxWeights),
                                        _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_aux_losses_workspace_bytes": (C.c_size_t, [C.POINTER(AuxDims)]),
    "dwa_aux_losses": (C.c_int, [_P, C.POINTER(AuxDims), C.POINTER(AuxWeights), _P, _P, _P, _P, _P, _P, _P,
                                 _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_bwd_workspace_bytes": (C.c_size_t, [C.POINTER(RetrieveDims), C.c_int]),
    "dwa_retrieve_bwd": (C.c_int, [_P, C.POINTER(RetrieveDims), C.c_int, C.c_int, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t]),
    "dwa_retrieve_merge": (C.c_int, [_P, C.POINTER(RetrieveDims), C.c_int, _P, C.c_int, _P, _P, _P,
                                     _P, _P, _P, C.c_size_t]),
}

_lib = None
_lock = threading.Lock()


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libdwa.so once; raise if it is missing or lacks a declared symbol."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise DwaError(f"{path} is missing: build it with `python -m matrix_b200.build`")
        lib = C.CDLL(path)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.dwa_abi_version() != 1:
            raise DwaError("libdwa ABI version mismatch")
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(1024)
    lib.dwa_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != DWA_OK:
        lib = load()
        raise DwaError(f"{what}: {lib.dwa_status_string(rc).decode()} ({rc}): {last_error()}")


def launch_counters() -> tuple[int, int, int]:
    lib = load()
    t, a, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.dwa_launch_counters(C.byref(t), C.byref(a), C.byref(b))
    return t.value, a.value, b.value


def describe_status(bits: int) -> str:
    return ", ".join(msg for bit, msg in STATUS_BITS.items() if bits & bit) or "ok"
