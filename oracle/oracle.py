"""numpy front end of the CPU oracle (oracle/qvex_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and by the
``cpu_baseline`` / ``--impl reference`` legs of bench.py, always as the checker or the
timed CPU baseline, never as the product path.

bf16 tensors are carried as ``uint16`` bit patterns (or ``ml_dtypes.bfloat16`` views);
each function names the reference arithmetic it restates (see the C file header).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    srcs = [HERE / "qvex_oracle.c", HERE / "model_oracle.c", HERE / "Makefile"]
    if force or not LIB_PATH.exists() or any(LIB_PATH.stat().st_mtime < s.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        L.orc_pack4.argtypes = [P, P, I64, I64]
        L.orc_unpack4.argtypes = [P, P, I64, I64]
        L.orc_quantize.argtypes = [P, I64, I64, I, I, P, P, P]
        L.orc_quantize.restype = I
        L.orc_dequantize.argtypes = [P, P, P, P, I64, I64, I]
        L.orc_qmm_exact.argtypes = [P, P, P, P, P, P, I64, I64, I64, I]
        L.orc_qmv_fast.argtypes = [P, P, P, P, P, I64, I64, I64, I64, I64]
        L.orc_gated_delta.argtypes = [P] * 11 + [I] * 6
        L.orc_gated_delta.restype = I
        L.orc_qk_condition.argtypes = [P, P, I64, I]
        L.orc_sample_scores.argtypes = [P, P, P, I64, I64, ctypes.c_float, ctypes.c_float, I, ctypes.c_float]
        L.orc_sample_scores.restype = I
        F = ctypes.c_float
        L.orc_rms_norm.argtypes = [P, P, P, F, P, P, I64, I, I]
        L.orc_gated_rms_norm.argtypes = [P, P, I64, P, F, P, I64, I, I]
        L.orc_swiglu.argtypes = [P, I64, P, I64, I64]
        L.orc_deltanet_conv.argtypes = [P, I64, P, P, P, P, P, P, P, P, P] + [I] * 7
        L.orc_attention.argtypes = [P, I64, P, P, F, P, I, P, P, I, I, P, I, I, I, I, I, F]
        L.orc_f32_to_bf16.argtypes = [P, P, I64]
        L.orc_bf16_to_f32.argtypes = [P, P, I64]
        L.orc_num_threads.restype = I
        L.orc_set_num_threads.argtypes = [I]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.c_void_p)


def _u16(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype != np.uint16:
        a = a.view(np.uint16) if a.dtype.itemsize == 2 else None
    return np.ascontiguousarray(a)


# ------------------------------------------------------------------ bf16 helpers

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = _u16(h)
    out = np.empty(h.shape, np.float32)
    lib().orc_bf16_to_f32(_p(h), _p(out), h.size)
    return out


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


# ------------------------------------------------------------------ format

def pack4(codes: np.ndarray) -> np.ndarray:
    """uint8 codes [N, K] -> uint32 [N, K/8] (quant/quantize.py:71-75 bit order)."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    N, K = codes.shape
    assert K % 8 == 0
    out = np.empty((N, K // 8), np.uint32)
    lib().orc_pack4(_p(codes), _p(out), N, K)
    return out


def unpack4(words: np.ndarray, K: int | None = None) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    N = words.shape[0]
    K = words.shape[1] * 8 if K is None else K
    out = np.empty((N, K), np.uint8)
    lib().orc_unpack4(_p(words), _p(out), N, K)
    return out


VARIANTS = {"minmax": 0, "zero_exact": 1}


def quantize(w_bf16: np.ndarray, group_size: int = 64, variant: str = "minmax"):
    """bf16 [N, K] -> (w uint32 [N, K/8], scales bf16 [N, K/gs], biases bf16 [N, K/gs])."""
    w = _u16(w_bf16)
    N, K = w.shape
    G = K // group_size
    wq = np.empty((N, K // 8), np.uint32)
    s = np.empty((N, G), np.uint16)
    b = np.empty((N, G), np.uint16)
    rc = lib().orc_quantize(_p(w), N, K, group_size, VARIANTS[variant], _p(wq), _p(s), _p(b))
    if rc != 0:
        raise ValueError("oracle quantize: unsupported arguments")
    return wq, s, b


def dequantize(wq, scales, biases, group_size: int = 64) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s, b = _u16(scales), _u16(biases)
    N = wq.shape[0]
    K = wq.shape[1] * 8
    out = np.empty((N, K), np.uint16)
    lib().orc_dequantize(_p(wq), _p(s), _p(b), _p(out), N, K, group_size)
    return out


def qmm_exact(x, wq, scales, biases, group_size: int = 64, want_f32: bool = False):
    """y bf16 [M, N] = x [M, K] @ dequant(w)^T with double accumulation."""
    x = _u16(x)
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s, b = _u16(scales), _u16(biases)
    M, K = x.shape
    N = wq.shape[0]
    assert wq.shape[1] * 8 == K
    y = np.empty((M, N), np.uint16)
    y32 = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_qmm_exact(_p(x), _p(wq), _p(s), _p(b), _p(y),
                        _p(y32) if want_f32 else None, M, N, K, group_size)
    return (y, y32) if want_f32 else y


def qmv_fast(x, wq, scales, biases, n0: int = 0, n1: int | None = None, out=None):
    """Reference multi-row matvec arithmetic (fp32), rows [n0, n1) of y bf16 [M, N]."""
    x = _u16(x)
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s, b = _u16(scales), _u16(biases)
    M, K = x.shape
    N = wq.shape[0]
    assert M <= 8 and K % 64 == 0
    y = np.zeros((M, N), np.uint16) if out is None else out
    lib().orc_qmv_fast(_p(x), _p(wq), _p(s), _p(b), _p(y), M, N, K, n0, N if n1 is None else n1)
    return y


def gated_delta(q, k, v, a, b, A_log, dt_bias, state, keep_mid: bool = False):
    """engine/kernels.py:92-116 semantics: returns (y, state_out[, state_mid])."""
    q, k, v, a, b = (_u16(t) for t in (q, k, v, a, b))
    A_log = np.ascontiguousarray(A_log, dtype=np.float32)
    dt_bias = np.ascontiguousarray(dt_bias, dtype=np.float32)
    state = np.ascontiguousarray(state, dtype=np.float32)
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2:]
    y = np.empty((B, T, Hv, Dv), np.uint16)
    so = np.empty_like(state)
    sm = np.empty_like(state) if keep_mid else None
    rc = lib().orc_gated_delta(_p(q), _p(k), _p(v), _p(a), _p(b), _p(A_log), _p(dt_bias),
                               _p(state), _p(y), _p(so), _p(sm) if keep_mid else None,
                               B, T, Hk, Hv, Dk, Dv)
    if rc != 0:
        raise ValueError("oracle gated_delta: unsupported shape")
    return (y, so, sm) if keep_mid else (y, so)


def qk_condition(q, k):
    """engine/model.py:275-277 on bf16 q, k [..., D] (returns new arrays)."""
    q = _u16(q).copy()
    k = _u16(k).copy()
    D = q.shape[-1]
    lib().orc_qk_condition(_p(q), _p(k), q.size // D, D)
    return q, k


def sample_scores(logits, seen=None, temperature=0.6, top_p=0.95, top_k=20, presence_penalty=0.0):
    """engine/sampler.py:30-62 (Sampler.scores) on fp32 logits [M, V]; seen [V] or None."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    M, V = x.shape
    out = np.empty_like(x)
    sn = None if seen is None else np.ascontiguousarray(seen, dtype=np.float32)
    rc = lib().orc_sample_scores(_p(x), _p(sn) if sn is not None else None, _p(out), M, V, temperature, top_p,
                                 top_k, presence_penalty)
    if rc:
        raise MemoryError("oracle sample_scores")
    return out


def threads_env() -> int:
    """Host threads this process may use (affinity mask)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ------------------------------------------------------------------ layer glue (model_oracle.c)

def rms_norm(x, w=None, eps: float = 1e-6, resid=None, chunk: int = 32):
    """mx.fast.rms_norm over the last axis (engine/model.py:314,316,335); with ``resid`` the
    residual add h = x + resid comes first.  Returns out (and h when resid is given)."""
    x = _u16(x)
    D = x.shape[-1]
    M = x.size // D
    out = np.empty(x.shape, np.uint16)
    h = np.empty(x.shape, np.uint16) if resid is not None else None
    r = _u16(resid) if resid is not None else None
    wv = _u16(w) if w is not None else None
    lib().orc_rms_norm(_p(x), _p(r) if r is not None else None, _p(wv) if wv is not None else None, eps,
                       _p(h) if h is not None else None, _p(out), M, D, chunk)
    return (out, h) if resid is not None else out


def gated_rms_norm(y, z, w, eps: float = 1e-6):
    """_gated_rmsnorm (engine/model.py:138-143): y [T, H, D], z [T, >= H*D] (row stride of
    its last axis), w [D] -> bf16 [T, H*D]."""
    y = _u16(y)
    T, H, D = y.shape
    z = _u16(z).reshape(T, -1)
    out = np.empty((T, H * D), np.uint16)
    lib().orc_gated_rms_norm(_p(y), _p(z), z.shape[1], _p(_u16(w)), eps, _p(out), T, H, D)
    return out


def swiglu(gu):
    """_swiglu (engine/model.py:133-135) on gu [M, 2I] = [gate | up] -> bf16 [M, I]."""
    gu = _u16(gu)
    M, I2 = gu.shape
    out = np.empty((M, I2 // 2), np.uint16)
    lib().orc_swiglu(_p(gu), I2, _p(out), M, I2 // 2)
    return out


def deltanet_conv(proj, conv_w, state, Hk, Hv, Dk, Dv, keep_mid: bool = False):
    """engine/model.py:259-277 up to the gated_delta call.  proj [B, T, >= C + Hv*Dv + 2Hv]
    (the in_proj output), conv_w fp32 [C, KW], state bf16 [B, KW-1, C].  Returns
    (q, k, v, a, b, state_out[, state_mid])."""
    proj = _u16(proj)
    B, T, S = proj.shape
    conv_w = np.ascontiguousarray(conv_w, dtype=np.float32)
    C, KW = conv_w.shape
    st = _u16(state)
    q = np.empty((B, T, Hk, Dk), np.uint16)
    k = np.empty_like(q)
    v = np.empty((B, T, Hv, Dv), np.uint16)
    a = np.empty((B, T, Hv), np.uint16)
    b = np.empty_like(a)
    so = np.empty((B, KW - 1, C), np.uint16)
    sm = np.empty_like(so) if keep_mid else None
    lib().orc_deltanet_conv(_p(proj), S, _p(conv_w), _p(st), _p(so), _p(sm) if keep_mid else None, _p(q), _p(k),
                            _p(v), _p(a), _p(b), B, T, Hk, Hv, Dk, Dv, KW)
    return (q, k, v, a, b, so, sm) if keep_mid else (q, k, v, a, b, so)


def rope_inv_freq(rd: int, base: float) -> np.ndarray:
    """fp32 rope frequencies base^(-2i/rd), i < rd/2, computed in double and rounded once."""
    i = np.arange(rd // 2, dtype=np.float64)
    return (base ** (-2.0 * i / rd)).astype(np.float32)


def attention(qkv, qn, kn, k_cache, v_cache, pos0: int, H: int, Hkv: int, D: int, rd: int, base: float,
              eps: float = 1e-6, scale: float | None = None):
    """Attention between its projections (engine/model.py:213-232).  qkv [B, L, H*2D +
    2*Hkv*D], caches bf16 [B, Hkv, cap, D] (updated in place at [pos0, pos0 + L)).
    Returns bf16 [B, L, H*D] (the o_proj input)."""
    qkv = _u16(qkv)
    B, L, S = qkv.shape
    cap = k_cache.shape[2]
    assert k_cache.dtype == np.uint16 and k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    out = np.empty((B, L, H * D), np.uint16)
    inv = rope_inv_freq(rd, base)
    lib().orc_attention(_p(qkv), S, _p(_u16(qn)), _p(_u16(kn)), eps, _p(inv), rd, _p(k_cache), _p(v_cache), cap,
                        pos0, _p(out), B, L, H, Hkv, D, D ** -0.5 if scale is None else scale)
    return out
