"""Loader for the in-tree C-ABI library `_oa_b200.so` (the only compute path of this package).

There is no fallback: if the library is missing or a call reports an error, the caller gets a
RuntimeError.  Argument types are declared once from the signatures in include/openattention_b200.h.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_oa_b200.so")
OA_BF16, OA_F32 = 0, 1

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes); every compute entry returns an int status.
SIGNATURES = {
    "oa_version": (ctypes.c_char_p, []),
    "oa_last_error_string": (ctypes.c_char_p, []),
    "oa_flash_workspace_bytes": (SZ, [I64, I64, I64, I64, I32]),
    "oa_flash_kvhead_proxies": (I32, [P, I64, P, P, I64, I64, P, I64, P, I64, P, P, I64, I64, P, I64, P, I64,
                                      I32, I64, I64, I64, I64, F32, I32, P, SZ, P]),
    "oa_flash_qhead_proxies": (I32, [P, I64, P, P, I64, I64, P, I64, P, I64, P, P, I64, I64, P, I64, P, I64,
                                     I32, I64, I64, I64, I64, F32, I32, P, SZ, P]),
    "oa_flash_qhead_proxies_noalloc": (I32, [P, I64, P, P, I64, I64, P, I64, P, I64, P, P, I64, I64, P, I64, P,
                                             I64, I32, I64, I64, I64, I64, F32, I32, P]),
    "oa_index_update": (I32, [P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, I32, P, I64, P, P,
                              P]),
    "oa_append_kv": (I32, [P, P, I64, I64, I64, P, P, P, I32, I32, P, P]),
    "oa_index_update_append": (I32, [P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I32,
                                     P, I64, P, P, P]),
    "oa_qgs_scan": (I32, [P, P, I64, I64, I64, P, I32, I32, P, I64, P, I64, P, P]),
    "oa_qgs_select": (I32, [P, I64, P, I64, I64, I64, P, I32, I32, I32, P, P]),
    "oa_errorgate_waterfill": (I32, [P, I64, P, I64, I64, I64, I64, P, P, I64, P, P, P, F32, P, P, P, P, P, P]),
    "oa_topq": (I32, [P, I64, I64, I64, I64, P, P, P, P, P, P, I32, P, I64, P, P, P, P, P, SZ, P]),
    "oa_topq_workspace_bytes": (SZ, [I64, I64, I64]),
    "oa_topq_variant": (I32, [I64, I64, I64]),
    "oa_residual": (I32, [P, P, I64, I64, I64, I64, P, P, I64, P, I64, P, P, P, P, P, P, P, P, P]),
    "oa_residual_flash": (I32, [P, I64, P, P, I64, I64, I64, I64, P, P, I64, P, I64, P, P, P, P, P, P, P, P, P,
                                I64, I32, F32, P, P]),
    "oa_build_codes": (I32, [P, I64, I64, I64, P, P, P, P, P]),
    "oa_build_project_workspace_bytes": (SZ, [I64]),
    "oa_build_project": (I32, [P, I64, I64, I64, P, P, P, P, SZ, P]),
    "oa_kmeans_assign": (I32, [P, I64, I64, I64, P, P, I64, P]),
    "oa_csr_workspace_bytes": (SZ, [I64, I64]),
    "oa_csr_build": (I32, [P, I64, I64, I64, I64, P, I64, P, P, P, SZ, P]),
    "oa_kmeans_update": (I32, [P, I64, I64, I64, P, I64, P, P, P, P, P, P]),
    "oa_cluster_sums": (I32, [P, P, I64, I64, I64, P, I64, P, P, P, P, P, P]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the library (once).  Raises RuntimeError when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m openattention_b200.build` "
                                   "(or __graft_entry__.build()); this package has no CPU fallback")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise RuntimeError with the library's message on failure."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.oa_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{name} failed (status {status}): {msg}")


def ptr(t) -> int:
    """Device pointer of a tensor (None -> NULL)."""
    return 0 if t is None else t.data_ptr()
