"""ctypes binding of libtarscuda.so (include/tarscuda.h).

The library is built in-tree by `python -m opentars_b200.build` (or __graft_entry__.build()).
There is no fallback: when the library or a CUDA device is missing, loading fails with an error.
"""
from __future__ import annotations

import ctypes
import functools
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtarscuda.so"

TC_OK, TC_CONTRACT, TC_ERR_CUDA, TC_ERR_ARG, TC_ERR_TOO_LARGE = 0, 1, -1, -2, -3
ABI_VERSION = 1


class Status_t(ctypes.Structure):
    _fields_ = [("done", ctypes.c_int32), ("err_code", ctypes.c_int32), ("op_idx", ctypes.c_int32)]


class OpStat_t(ctypes.Structure):
    _fields_ = [("opcode", ctypes.c_uint64), ("macs", ctypes.c_uint64), ("bytes_read", ctypes.c_uint64),
                ("bytes_written", ctypes.c_uint64)]


class Seg_t(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("base_lo", ctypes.c_uint64), ("base_hi", ctypes.c_uint64),
                ("ld", ctypes.c_uint64), ("nbytes", ctypes.c_uint64), ("count", ctypes.c_uint64)]


# name: (restype, argtypes) for every entry point include/tarscuda.h declares
P, U8P, VP = ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.c_void_p
SIGNATURES = {
    "tc_version": (ctypes.c_int, []),
    "tc_open": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "tc_close": (ctypes.c_int, [P]),
    "tc_last_error": (ctypes.c_char_p, [P]),
    "tc_device_ptr": (ctypes.c_uint64, [P]),
    "tc_stream": (ctypes.c_void_p, [P]),
    "tc_upload": (ctypes.c_int, [P, ctypes.c_uint64, VP, ctypes.c_uint64]),
    "tc_download": (ctypes.c_int, [P, ctypes.c_uint64, VP, ctypes.c_uint64]),
    "tc_sync_up": (ctypes.c_int, [P, VP, VP, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "tc_sync_down": (ctypes.c_int, [P, VP, VP]),
    "tc_run_queue": (ctypes.c_int, [P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32,
                                    ctypes.POINTER(Status_t), ctypes.POINTER(ctypes.c_int32)]),
    "tc_stats": (ctypes.c_uint32, [P, ctypes.POINTER(OpStat_t), ctypes.c_uint32]),
    "tc_validate": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64)]),
    "tc_footprint": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(Seg_t), ctypes.c_uint32,
                                    ctypes.POINTER(ctypes.c_uint32)]),
    "tc_queue_capture": (ctypes.c_int, [P, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.POINTER(Status_t), ctypes.POINTER(ctypes.c_int32),
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "tc_graph_launch": (ctypes.c_int, [P, VP]),
    "tc_graph_times": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_float), ctypes.c_uint32]),
    "tc_graph_destroy": (ctypes.c_int, [P]),
    "tc_graph_kernels": (ctypes.c_int, [P]),
    "tc_synchronize": (ctypes.c_int, [P]),
    "tc_set_mma_min_rows": (ctypes.c_int, [ctypes.c_int32]),
    "tc_mma_trace": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint32]),
    "tc_wait_error": (ctypes.c_int, [ctypes.c_int32]),
    "tc_set_spin_limit": (ctypes.c_uint32, [ctypes.c_uint32]),
    "tc_conv_w8a8_noalloc": (ctypes.c_int, [VP, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, VP, VP,
                                            ctypes.c_int32, VP, VP, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_float, VP]),
}


class LibraryMissing(RuntimeError):
    pass


@functools.lru_cache(None)
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise LibraryMissing(f"{LIB_PATH} is not built: run `python -m opentars_b200.build`")
    L = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
    if L.tc_version() != ABI_VERSION:
        raise LibraryMissing(f"{LIB_PATH}: ABI {L.tc_version()}, this package needs {ABI_VERSION}")
    return L


def check(rc: int, handle=None, what: str = "") -> int:
    if rc < 0:
        msg = lib().tc_last_error(handle).decode() if handle else ""
        raise RuntimeError(f"libtarscuda {what} failed ({rc}): {msg}")
    return rc
