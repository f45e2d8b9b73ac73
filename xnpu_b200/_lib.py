"""ctypes binding of libxq4.so (the C ABI declared in include/xq4.h).

The shared library is built in-tree (``python xnpu_b200/build.py``) and loaded
from this package directory.  There is no fallback: if the library is missing,
every entry point of the package raises.
"""
import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libxq4.so"

XQ4_OK = 0
XQ4_EINVAL = 1
XQ4_ENOMEM = 2
XQ4_ECUDA = 3
XQ4_ETIMEDOUT = 4
XQ4_ENCCL = 5
XQ4_ENOTSUP = 6
XQ4_ENODEV = 7

XQ4_LAYOUT_L1 = 1
XQ4_LAYOUT_L2 = 2
XQ4_LAYOUT_PLANES = 3
XQ4_CODE_S4 = 0
XQ4_CODE_U4_ZP8 = 1
XQ4_SCALE_BF16 = 0
XQ4_SCALE_FP16 = 1
XQ4_OUT_BF16 = 0
XQ4_OUT_F32 = 1
XQ4_UNIQUE_ID_BYTES = 128
XQ4_NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024  # include/xq4.h
XQ4_FUSED_MAX_VALUES = 4 * 1024 * 1024  # include/xq4.h

_STATUS_NAMES = {
    XQ4_OK: "XQ4_OK", XQ4_EINVAL: "XQ4_EINVAL", XQ4_ENOMEM: "XQ4_ENOMEM", XQ4_ECUDA: "XQ4_ECUDA",
    XQ4_ETIMEDOUT: "XQ4_ETIMEDOUT", XQ4_ENCCL: "XQ4_ENCCL", XQ4_ENOTSUP: "XQ4_ENOTSUP",
    XQ4_ENODEV: "XQ4_ENODEV",
}


class Xq4Error(OSError):
    """A libxq4 call failed; ``status`` is the XQ4_* code."""

    def __init__(self, status, message):
        super().__init__(status, f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class LayoutDesc(ctypes.Structure):
    _fields_ = [
        ("layout", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int), ("group", ctypes.c_int),
        ("tsi", ctypes.c_int), ("cols", ctypes.c_int), ("code_format", ctypes.c_int),
        ("scale_dtype", ctypes.c_int), ("scale_offset", ctypes.c_size_t),
        ("row_begin", ctypes.c_int), ("row_end", ctypes.c_int),
    ]


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("ordinal", ctypes.c_int), ("sm_count", ctypes.c_int), ("cc_major", ctypes.c_int),
        ("cc_minor", ctypes.c_int), ("hbm_bytes", ctypes.c_size_t), ("l2_bytes", ctypes.c_size_t),
        ("name", ctypes.c_char * 96),
    ]


class ChainOp(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p), ("x_dev", ctypes.c_void_p), ("y_dev", ctypes.c_void_p),
        ("m", ctypes.c_int), ("out_dtype", ctypes.c_int), ("wait_prev", ctypes.c_int),
        ("comm", ctypes.c_void_p),
        ("norm_w_dev", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("residual_dev", ctypes.c_void_p),
        ("swiglu", ctypes.c_int), ("w4a8", ctypes.c_int),
    ]


_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_I = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); one line per declaration of include/xq4.h
SIGNATURES = {
    "xq4_last_error_string": (ctypes.c_char_p, []),
    "xq4_version": (ctypes.c_char_p, []),
    "xq4_device_open": (_I, [_I, _PP]),
    "xq4_device_close": (_I, [_P]),
    "xq4_device_query": (_I, [_P, ctypes.POINTER(DeviceInfo)]),
    "xq4_device_stream": (_P, [_P]),
    "xq4_buffer_create": (_I, [_P, _SZ, _PP]),
    "xq4_buffer_upload": (_I, [_P, _P, _SZ, _SZ]),
    "xq4_buffer_download": (_I, [_P, _P, _SZ, _SZ]),
    "xq4_buffer_destroy": (_I, [_P]),
    "xq4_buffer_device_ptr": (_P, [_P]),
    "xq4_buffer_size": (_SZ, [_P]),
    "xq4_weight_import": (_I, [_P, _P, _SZ, ctypes.POINTER(LayoutDesc), _PP]),
    "xq4_weight_destroy": (_I, [_P]),
    "xq4_weight_shape": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_SZ)]),
    "xq4_gpu_layout_bytes": (_SZ, [_I, _I]),
    "xq4_repack_host": (_I, [_P, _SZ, ctypes.POINTER(LayoutDesc), _P, _SZ]),
    "xq4_dequant": (_I, [_P, _P, _P]),
    "xq4_linear": (_I, [_P, _P, _P, _SZ, _P, _SZ, _I, _I, ctypes.POINTER(ctypes.c_uint64)]),
    "xq4_linear_raw": (_I, [_P, _P, _P, _I, _I, _P]),
    "xq4_chain_create": (_I, [_P, ctypes.POINTER(ChainOp), _I, _PP]),
    "xq4_chain_destroy": (_I, [_P]),
    "xq4_chain_submit": (_I, [_P, _P, ctypes.POINTER(ctypes.c_uint64)]),
    "xq4_chain_run": (_I, [_P, _P]),
    "xq4_wait": (_I, [_P, ctypes.c_uint64, ctypes.c_int64]),
    "xq4_last_seq": (ctypes.c_uint64, [_P]),
    "xq4_device_fault": (_I, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "xq4_comm_unique_id": (_I, [_P]),
    "xq4_comm_init": (_I, [_P, _I, _I, _P, _PP]),
    "xq4_comm_destroy": (_I, [_P]),
    "xq4_linear_sharded": (_I, [_P, _P, _P, _P, _P, _I, _I, _P]),
    "xq4_linear_sharded_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "xq4_linear_sharded_fused": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "xq4_quantize_x": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "xq4_linear_w4a8": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "xq4_attn_create": (_I, [_P, _I, _I, _I, ctypes.c_float, _PP]),
    "xq4_attn_destroy": (_I, [_P]),
    "xq4_attn_decode": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P]),
}

_lib = None


def lib():
    """Load libxq4.so once; raise if it is missing (no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python xnpu_b200/build.py` "
                "(the int4 path has no CPU fallback)")
        L = ctypes.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error():
    return lib().xq4_last_error_string().decode(errors="replace")


def check(status):
    """Raise Xq4Error for a non-zero status."""
    if status != XQ4_OK:
        raise Xq4Error(status, last_error())
    return status
