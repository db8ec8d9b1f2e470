"""ctypes binding of ``libflash_spacetime.so`` (the C ABI in include/flash_spacetime.h).

The structures below mirror the C structs field for field. The library is
loaded from this package's folder; if it is missing the op raises instead
of falling back to anything else.
"""

import ctypes
import os
import threading
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflash_spacetime.so")

FST_F32, FST_BF16, FST_F16 = 0, 1, 2
FST_OK = 0
FST_ERR_INVALID = 1
FST_ERR_UNSUPPORTED = 2
FST_ERR_CUDA = 3
FST_ERR_WORKSPACE = 4
FST_ERR_DEVICE = 5

ABI_VERSION = 5
FST_FLAG_SHARE_SMS = 1  # FstProblem.flags: another kernel shares the SMs
FST_FLAG_LONGEST_FIRST = 2  # FstProblem.flags: the library orders the events itself
MAX_SELF_ORDERED = 1024  # events FST_FLAG_LONGEST_FIRST accepts

EXPORTED = (
    "fst_abi_version",
    "fst_forward_workspace_size",
    "fst_backward_workspace_size",
    "fst_dw_partial_count",
    "fst_sum_partials",
    "fst_forward",
    "fst_backward",
    "fst_forward_noalloc",
    "fst_upload_rows",
    "fst_kernel_launches",
    "fst_last_error",
)


class FstProblem(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("packed", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("max_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("feat_stride", ctypes.c_int32),
        ("total_rows", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("use_attn_bias", ctypes.c_int32),
        ("use_act_bias", ctypes.c_int32),
        ("seqlens", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("feats", ctypes.c_void_p),
        ("freqs", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("event_order", ctypes.c_void_p),
        ("qkv_row_stride", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("valid_rows", ctypes.c_int64),
    ]


class FstForwardArgs(ctypes.Structure):
    _fields_ = [
        ("prob", FstProblem),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("u", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class FstBackwardArgs(ctypes.Structure):
    _fields_ = [
        ("prob", FstProblem),
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("u", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("dout", ctypes.c_void_p),
        ("wt", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("dw_partial", ctypes.c_void_p),
        ("db_partial", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("sigma", ctypes.c_void_p),
        ("ds_absmax", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is missing or stale."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"flash_spacetime: {LIB_PATH} is missing; build it with "
                "`make -C flash-spacetime_b200` (there is no fallback path)"
            )
        lib = ctypes.CDLL(LIB_PATH)
        lib.fst_abi_version.restype = ctypes.c_int
        lib.fst_forward_workspace_size.restype = ctypes.c_size_t
        lib.fst_forward_workspace_size.argtypes = [ctypes.POINTER(FstProblem)]
        lib.fst_backward_workspace_size.restype = ctypes.c_size_t
        lib.fst_backward_workspace_size.argtypes = [ctypes.POINTER(FstProblem)]
        lib.fst_dw_partial_count.restype = ctypes.c_int64
        lib.fst_dw_partial_count.argtypes = [ctypes.POINTER(FstProblem)]
        lib.fst_sum_partials.restype = ctypes.c_int
        lib.fst_sum_partials.argtypes = [ctypes.POINTER(FstProblem), ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p]
        lib.fst_forward.restype = ctypes.c_int
        lib.fst_forward.argtypes = [ctypes.POINTER(FstForwardArgs), ctypes.c_void_p]
        lib.fst_backward.restype = ctypes.c_int
        lib.fst_backward.argtypes = [ctypes.POINTER(FstBackwardArgs), ctypes.c_void_p]
        lib.fst_forward_noalloc.restype = ctypes.c_int
        lib.fst_forward_noalloc.argtypes = [ctypes.POINTER(FstForwardArgs), ctypes.c_void_p]
        lib.fst_upload_rows.restype = ctypes.c_int
        lib.fst_upload_rows.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_void_p]
        lib.fst_kernel_launches.restype = ctypes.c_int64
        lib.fst_last_error.restype = ctypes.c_int
        lib.fst_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        got = lib.fst_abi_version()
        if got != ABI_VERSION:
            raise RuntimeError(f"libflash_spacetime ABI {got} != expected {ABI_VERSION}")
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().fst_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Raise the Python error matching a C status code."""
    if rc == FST_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (FST_ERR_INVALID, FST_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)
