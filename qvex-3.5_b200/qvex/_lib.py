"""ctypes binding of libqvex.so (declarations in include/qvex.h).

The library is the only compute path: if it is missing or fails to load, every call
raises.  There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libqvex.so")

QVX_OK = 0
QVX_ERR_INVALID = 1
QVX_ERR_UNSUPPORTED = 2
QVX_ERR_ALIGN = 3
QVX_ERR_CUDA = 4
QVX_ERR_TIMEOUT = 5
QVX_ERR_WORKSPACE = 6

QVX_QUANT_MINMAX = 0
QVX_QUANT_ZERO_EXACT = 1

# Every entry point of include/qvex.h: name -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
SIGNATURES = {
    "qvx_version": (_I, []),
    "qvx_last_error": (ctypes.c_char_p, []),
    "qvx_device_status": (_I, [_P, ctypes.POINTER(_I)]),
    "qvx_qmv": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "qvx_qmm_workspace_size": (_SZ, [_I, _I, _I]),
    "qvx_qmm": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "qvx_qmm_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "qvx_qmm_prepared_bytes": (_SZ, [_I, _I]),
    "qvx_qmm_prepare": (_I, [_P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "qvx_qmm_prepared": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "qvx_qmv_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "qvx_qmv_fused": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "qvx_quantized_matmul": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "qvx_quantize": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "qvx_dequantize": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "qvx_dequantize_rows": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "qvx_gated_delta": (_I, [_P] * 11 + [_I] * 6 + [_P]),
    "qvx_qk_condition": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _I, _P]),
    "qvx_rms_norm": (_I, [_P, _P, _P, ctypes.c_float, _P, _P, ctypes.c_longlong, _I, _P]),
    "qvx_add": (_I, [_P, _P, _P, ctypes.c_longlong, _P]),
    "qvx_gated_rms_norm": (_I, [_P, _P, ctypes.c_longlong, _P, ctypes.c_float, _P, ctypes.c_longlong, _I, _I, _P]),
    "qvx_swiglu": (_I, [_P, ctypes.c_longlong, _P, ctypes.c_longlong, ctypes.c_longlong, _P]),
    "qvx_swiglu_pairs": (_I, [_P, ctypes.c_longlong, _P, ctypes.c_longlong, ctypes.c_longlong, _P]),
    "qvx_deltanet_conv": (_I, [_P, ctypes.c_longlong, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P] + [_I] * 6 + [_P]),
    "qvx_deltanet_decode": (_I, [_P, ctypes.c_longlong, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_float, _P]
                            + [_I] * 6 + [_P]),
    "qvx_attention_workspace_size": (_SZ, [_I] * 6),
    "qvx_attention": (_I, [_P, ctypes.c_longlong, _P, _P, ctypes.c_float, _P, _I, _P, _P, _I, _P, _I, _P, _P]
                      + [_I] * 5 + [ctypes.c_float, _P, _SZ, _I, _P]),
    "qvx_sample_scores": (_I, [_P, _I, _P, _P, _I, _I, ctypes.c_float, ctypes.c_float, _I, ctypes.c_float, _P]),
    "qvx_sample_pick": (_I, [_P, _P, _I, _I, _I, ctypes.c_ulonglong, ctypes.c_ulonglong, _P]),
}


QVX_MAX_RANKS = 8


class QvxGather(ctypes.Structure):
    """Mirror of ``qvx_gather`` (include/qvex.h): the output buffers and receive areas
    (inboxes) of a column-sharded projection, this rank's launch counters, and its place in
    the rows."""
    _fields_ = [("out", _P * QVX_MAX_RANKS), ("inbox", _P * QVX_MAX_RANKS), ("epoch", _P),
                ("world", _I), ("rank", _I), ("n_total", _I), ("row0", _I), ("slot", _I), ("mode", _I)]


QVX_EXCHANGE_GATHER = 0
QVX_EXCHANGE_REDUCE = 1
QVX_IN_PLAIN, QVX_IN_RMS_NORM, QVX_IN_SWIGLU, QVX_IN_GATED_RMS_NORM = 0, 1, 2, 3
QVX_OUT_PLAIN, QVX_OUT_SWIGLU_PAIRS = 0, 1  # enum qvx_qmv_epilogue


class QvxQmvIO(ctypes.Structure):
    """Mirror of ``qvx_qmv_io`` (include/qvex.h): the prologue and epilogue of a fused
    decode projection."""
    _fields_ = [("prologue", _I), ("x_stride", ctypes.c_longlong), ("norm_w", _P), ("z", _P),
                ("z_stride", ctypes.c_longlong), ("head_dim", _I), ("eps", ctypes.c_float), ("resid", _P),
                ("epilogue", _I)]


class QvexError(RuntimeError):
    """A libqvex call failed; ``code`` is the qvx_status value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class QvexTimeout(QvexError, TimeoutError):
    pass


_lib = None


def lib() -> ctypes.CDLL:
    """Load libqvex.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m qvex.build` in qvex-3.5_b200/ "
                              "(or __graft_entry__.build()). There is no fallback path.")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc == QVX_OK:
        return
    msg = lib().qvx_last_error().decode(errors="replace") or what
    if rc in (QVX_ERR_INVALID, QVX_ERR_ALIGN, QVX_ERR_WORKSPACE):
        raise ValueError(msg)
    if rc == QVX_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == QVX_ERR_TIMEOUT:
        raise QvexTimeout(rc, msg)
    raise QvexError(rc, msg)


def device_status(stream_handle: int) -> int:
    """Reads and clears the device status word (synchronises the stream)."""
    st = _I(0)
    check(lib().qvx_device_status(_P(stream_handle), ctypes.byref(st)), "qvx_device_status")
    return st.value
