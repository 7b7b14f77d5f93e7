"""ctypes binding of libparis_moe.so (the C ABI in include/paris_moe.h).

There is no fallback: if the library is missing or fails to load, every
operator raises.  ``load()`` never builds; ``build.py`` (or
``__graft_entry__.build()``) does.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libparis_moe.so")

# Every symbol include/paris_moe.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
SIGNATURES = {
    "pmoe_status_string": (ctypes.c_char_p, [_I]),
    "pmoe_version": (ctypes.c_char_p, []),
    "pmoe_workspace_size": (_I, [_I, _I, _I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "pmoe_route": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "pmoe_route_diag": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, ctypes.POINTER(ctypes.c_float),
                             ctypes.POINTER(_I), _P, _SZ, _P]),
    "pmoe_exact_logits": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "pmoe_block_forward": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P,
                                _I, _I, _I, _P, _P, _SZ, _P]),
    "pmoe_block_forward_profiled": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                                         _P, _I, _I, _I, _P, _P, _SZ, _P,
                                         ctypes.POINTER(_P), _I]),
    "pmoe_block_forward_noalloc": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                                        _P, _I, _I, _I, _P, _P]),
    "pmoe_noalloc_scratch_bytes": (_SZ, []),
    "pmoe_ep_buffer_bytes": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "pmoe_block_forward_ep": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P,
                                   _I, _I, _I, _I, _I, ctypes.POINTER(_P), _SZ, _I, _I, _I,
                                   _P, _P, _SZ, _P]),
    "pmoe_layer_forward": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, ctypes.c_float, _P, _P, _P, _P,
                                _P, _P, _P, _I, _I, _I, _I, _I, ctypes.POINTER(_P), _SZ, _I,
                                _I, _I, _P, _P, _SZ, _P]),
    "pmoe_rmsnorm": (_I, [_P, _I, _I, _P, ctypes.c_float, _P, _P]),
    "pmoe_rows_buffer_bytes": (_I, [_I, _I, ctypes.POINTER(_SZ)]),
    "pmoe_rows_partial": (_I, [_P, _I, _I, _I, ctypes.POINTER(_P)]),
    "pmoe_rows_allreduce": (_I, [ctypes.POINTER(_P), _I, _I, _I, _I, _I, _I, _P, _P]),
    "pmoe_rows_status": (_I, [_P, ctypes.POINTER(_I)]),
    "pmoe_ep_status_async": (_I, [_P, _P, _P]),
    "pmoe_rows_status_async": (_I, [_P, _P, _P]),
    "pmoe_route_slice": (_I, [_P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _SZ,
                              _P]),
    "pmoe_block_forward_rows": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P,
                                     _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "pmoe_rows_fused_buffer_bytes": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "pmoe_block_forward_rows_fused": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                                           _P, _I, _I, ctypes.POINTER(_P), _I, _I, _I, _P, _P,
                                           _SZ, _P,
                                           ctypes.POINTER(_P), _I]),
    "pmoe_block_forward_rows_profiled": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P,
                                              _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P,
                                              _SZ, _P, ctypes.POINTER(_P), _I]),
    "pmoe_read_status": (_I, [_P, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "pmoe_comm_create": (_I, [_I, _I, ctypes.POINTER(_P)]),
    "pmoe_comm_destroy": (_I, [_P]),
    "pmoe_comm_set_ep": (_I, [_P, ctypes.POINTER(_P), _SZ, _I]),
    "pmoe_comm_set_rows": (_I, [_P, ctypes.POINTER(_P), _I]),
    "pmoe_comm_next_rows_epoch": (_I, [_P, ctypes.POINTER(_I)]),
    "pmoe_comm_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                            ctypes.POINTER(_I)]),
    "pmoe_block_forward_comm": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P,
                                     _I, _P, _P, _SZ, _P, ctypes.POINTER(_P), _I]),
    "pmoe_ipc_alloc": (_I, [_SZ, ctypes.POINTER(_P)]),
    "pmoe_ipc_free": (_I, [_P]),
    "pmoe_ipc_handle": (_I, [_P, ctypes.c_char_p]),
    "pmoe_ipc_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "pmoe_ipc_close": (_I, [_P]),
}

PMOE_ERR_PEER_TIMEOUT = -6
PMOE_ERR_COMM_CAPACITY = -9

PMOE_F_SHARED = 1
PMOE_F_ROUTED = 2
PMOE_F_FORCE_STREAM = 4
PMOE_F_FORCE_TC = 8
PMOE_F_ROUTE_SLICE = 16

_lock = threading.Lock()
_lib = None


class PmoeError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: status {status} ({msg})")
        self.status = status


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python {_PKG}/build.py` "
                "(the MoE operator has no CPU or Python fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(fn_name: str, status: int) -> None:
    if status != 0:
        msg = load().pmoe_status_string(status).decode()
        raise PmoeError(fn_name, status, msg)


def workspace_size(T, H, E, K, I, Is) -> int:
    out = ctypes.c_size_t(0)
    check("pmoe_workspace_size", load().pmoe_workspace_size(T, H, E, K, I, Is, ctypes.byref(out)))
    return int(out.value)
