"""ctypes binding of the C ABI declared in include/polarquant_b200.h.

The shared library is built in-tree (``python -m polarquant_b200.build``) as
``polarquant_b200/_lib/libpolarquant_b200.so``.  There is no fallback: if the
library is missing, or no CUDA device is present, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libpolarquant_b200.so")

PQ_TOPK_MAX = 2048

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_Z = ctypes.c_size_t

# name -> (restype, argtypes); must list every symbol of the public header.
SIGNATURES = {
    "pq_version": (_I, []),
    "pq_last_error": (ctypes.c_char_p, []),
    "pq_device_status": (_I, [ctypes.POINTER(_I)]),
    "pq_selftest_wait_timeout": (_I, [_L, _P]),
    "pq_row_bytes": (_L, [_I, _I]),
    "pq_launch_count": (_L, []),
    "pq_rotate": (_I, [_P, _L, _I, _P, _P, _P]),
    "pq_rotation_planes_bytes": (_Z, [_I]),
    "pq_prepare_rotation": (_I, [_P, _I, _P, _Z, _P]),
    "pq_encode_workspace_bytes": (_Z, [_L, _I]),
    "pq_encode": (_I, [_P, _L, _I, _P, _P, _P, _I, _P, _L, _P, _P, _Z, _P]),
    "pq_rotate_tc": (_I, [_P, _L, _I, _P, _P, _P, _Z, _P]),
    "pq_decode_workspace_bytes": (_Z, [_L, _I]),
    "pq_decode": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _P, _P, _P, _Z, _P]),
    "pq_adc_scan_workspace_bytes": (_Z, [_L, _I, _I, _I]),
    "pq_adc_scan_kernel": (_I, [_L, _I, _I, _I, _I, _I, _L]),
    "pq_adc_batch_workspace_bytes": (_Z, [_L, _I, _I, _I]),
    "pq_adc_batch_kernel": (_I, [_L, _I, _I, _I, _I, _L]),
    "pq_adc_scan_noalloc_scratch_bytes": (_Z, []),
    "pq_adc_scan_noalloc": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P, _I, _L, _P, _P, _P]),
    "pq_adc_batch": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P, _I, _L, _P, _P, _P, _Z, _P]),
    "pq_adc_scan": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P, _I, _L, _P, _P, _P, _Z, _P]),
    "pq_twostage_workspace_bytes": (_Z, [_L, _I, _I, _I]),
    "pq_twostage": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P, _P, _I, _I, _L, _P, _P, _P,
                         _Z, _P]),
    "pq_rerank": (_I, [_P, _L, _P, _L, _I, _I, _P, _I, _P, _P, _I, _I, _L, _P, _P, _P]),
    "pq_topk_merge": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "pq_ivf_cell_ids": (_I, [_P, _L, _L, _I, _I, _I, _I, _P, _P, _P]),
    "pq_ivf_probe": (_I, [_P, _I, _I, _I, _I, _P, _I, _P, _P, _P]),
    "pq_ivf_workspace_bytes": (_Z, [_L, _I, _I, _I, _I]),
    "pq_ivf_csr_workspace_bytes": (_Z, [_L, _I]),
    "pq_ivf_build_csr": (_I, [_P, _L, _I, _P, _P, _P, _L, _P, _P, _P, _P, _Z, _P]),
    "pq_ivf_search": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _I, _P, _P, _I, _I, _P, _P, _P, _P,
                           _P, _I, _I, _I, _I, _I, _P, _P, _P, _Z, _P]),
    "pq_hamming_workspace_bytes": (_Z, [_L, _I, _I]),
    "pq_hamming_scan": (_I, [_P, _L, _L, _I, _P, _I, _I, _L, _P, _P, _P, _Z, _P]),
    "pq_hamming_twostage": (_I, [_P, _L, _P, _L, _P, _L, _I, _I, _P, _I, _P, _I, _I, _L, _P, _P,
                                 _P, _Z, _P]),
    "pq_unpack_rows": (_I, [_P, _L, _L, _I, _I, _I, _P, _P]),
    "pq_unpack_at": (_I, [_P, _L, _P, _L, _I, _I, _I, _P, _P]),
    "pq_repack": (_I, [_P, _L, _L, _I, _I, _I, _P, _L, _P]),
    "pq_pack_codes": (_I, [_P, _L, _I, _I, _P, _L, _P]),
}

_lock = threading.Lock()
_lib = None


class PQError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name} failed ({code}): {msg}")
        self.code = code


def load():
    """Loads the library once and declares every signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"polarquant_b200 CUDA library not built ({LIB_PATH} missing); "
                "run `python -m polarquant_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises PQError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.pq_last_error()
        raise PQError(name, rc, msg.decode() if msg else "")


def query(name: str, *args):
    """Calls a value-returning entry point (sizes, row bytes, version)."""
    return getattr(load(), name)(*args)


def device_status() -> int:
    """Synchronises the device and returns (and clears) the device error word."""
    code = _I(0)
    call("pq_device_status", ctypes.byref(code))
    return code.value
