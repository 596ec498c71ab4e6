"""Quantized ops with MLX's call surface, on CUDA tensors.

``quantized_matmul``, ``quantize`` and ``dequantize`` keep the argument names and
meaning of ``mx.quantized_matmul`` / ``mx.quantize`` / ``mx.dequantize`` as the
reference calls them (engine/model.py:87-91,127; tools/fetch_mtp.py:99;
bench/qmv_kernel_bench.py:14).  Tensors are torch CUDA tensors; packed weights are
uint32 (int32 is accepted as the same bits).  Outputs are freshly allocated; inputs are
never written.  Every op runs a libqvex kernel on the current CUDA stream; there is no
other path.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import _P, check, lib

SUPPORTED_BITS = (4,)
SUPPORTED_GROUP_SIZES = (64,)
QMV_MAX_M = 8
# With a prepared weight (qmm_prepare) the tensor-core path takes M >= QMM_MIN_M_PREPARED:
# qmv runs token pairs as separate CTA groups that each stream the whole weight, so from 5
# rows on the tensor-core kernel, which streams it once, is faster (M = 8 over the 9B
# decode shapes: 1329 against 980 GB/s; M = 4: 1375 against 1746).
QMM_MIN_M_PREPARED = 5


def _stream(t: torch.Tensor) -> _P:
    return _P(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> _P:
    return _P(t.data_ptr() if t is not None else 0)


def _require_cuda(name: str, t: torch.Tensor, dtypes) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libqvex has no CPU path)")
    if t.dtype not in dtypes:
        raise TypeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")


def _check_qparams(group_size: int, bits: int) -> None:
    if bits not in SUPPORTED_BITS or group_size not in SUPPORTED_GROUP_SIZES:
        raise NotImplementedError(
            f"only bits={SUPPORTED_BITS} with group_size={SUPPORTED_GROUP_SIZES} is implemented "
            f"(got bits={bits}, group_size={group_size})")


def _packed(w: torch.Tensor) -> torch.Tensor:
    _require_cuda("w", w, (torch.uint32, torch.int32))
    return w.contiguous()


def qmm_workspace_size(M: int, N: int, K: int) -> int:
    return int(lib().qvx_qmm_workspace_size(M, N, K))


def qmm_prepare(scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """The tensor-core kernel's weight prepass (per-row exponents, per-group fp16
    multipliers) of a constant weight, made once: a uint8 device buffer to pass to
    quantized_matmul as ``prep``."""
    _check_qparams(group_size, bits)
    _require_cuda("scales", scales, (torch.bfloat16,))
    _require_cuda("biases", biases, (torch.bfloat16,))
    if scales.dim() != 2 or tuple(biases.shape) != tuple(scales.shape):
        raise ValueError("scales and biases must be 2-D of one shape")
    N, G = scales.shape
    K = G * group_size
    scales = scales.contiguous()
    biases = biases.contiguous()
    nbytes = int(lib().qvx_qmm_prepared_bytes(N, K))
    prep = torch.empty(nbytes, dtype=torch.uint8, device=scales.device)
    check(lib().qvx_qmm_prepare(_ptr(scales), _ptr(biases), N, K, group_size, bits, _ptr(prep), nbytes,
                                _stream(scales)), "qvx_qmm_prepare")
    return prep


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4, *,
                     out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None,
                     prep: torch.Tensor | None = None) -> torch.Tensor:
    """y[..., N] = x[..., K] @ dequant(w)^T (mx.quantized_matmul with transpose=True).

    M = prod(x.shape[:-1]) <= 8 runs the SIMT decode kernel, larger M the tcgen05
    tensor-core kernel (which needs a workspace; one is taken from the caching
    allocator when none is given).  ``prep`` (from qmm_prepare of these scales and
    biases) spares the tensor-core path its per-call weight prepass (same results) and
    sends M >= QMM_MIN_M_PREPARED to it as well.
    """
    _check_qparams(group_size, bits)
    if not transpose:
        raise NotImplementedError("transpose=False is not on the QVex hot path (QLinear uses transpose=True)")
    _require_cuda("x", x, (torch.bfloat16,))
    w = _packed(w)
    _require_cuda("scales", scales, (torch.bfloat16,))
    _require_cuda("biases", biases, (torch.bfloat16,))
    if w.dim() != 2 or scales.dim() != 2 or biases.dim() != 2:
        raise ValueError("w, scales and biases must be 2-D")
    N, KW = w.shape
    K = KW * 32 // bits
    if x.shape[-1] != K:
        raise ValueError(f"x has last dim {x.shape[-1]} but w holds K={K}")
    G = K // group_size
    if tuple(scales.shape) != (N, G) or tuple(biases.shape) != (N, G):
        raise ValueError(f"scales/biases must be [{N}, {G}], got {tuple(scales.shape)} / {tuple(biases.shape)}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N), dtype=torch.bfloat16, device=x.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (*lead, N) or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor of shape x.shape[:-1] + (N,)")
    if M == 0:
        return out
    scales = scales.contiguous()
    biases = biases.contiguous()
    s = _stream(x2)
    if M <= QMV_MAX_M and (prep is None or M < QMM_MIN_M_PREPARED):
        check(lib().qvx_qmv(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size,
                            bits, s), "qvx_qmv")
    else:
        need = qmm_workspace_size(M, N, K)
        if workspace is None:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        if prep is not None:
            if prep.dtype != torch.uint8 or prep.device != x.device or prep.numel() < int(
                    lib().qvx_qmm_prepared_bytes(N, K)):
                raise ValueError("prep must be qmm_prepare's buffer for this weight, on x's device")
            check(lib().qvx_qmm_prepared(_ptr(x2), _ptr(w), _ptr(prep), _ptr(out), M, N, K, group_size, bits,
                                         _ptr(workspace), workspace.numel() * workspace.element_size(), s),
                  "qvx_qmm_prepared")
        else:
            check(lib().qvx_qmm(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size,
                                bits, _ptr(workspace), workspace.numel() * workspace.element_size(), s),
                  "qvx_qmm")
    return out


_VARIANTS = {"minmax": _lib.QVX_QUANT_MINMAX, "zero_exact": _lib.QVX_QUANT_ZERO_EXACT}


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, *, variant: str = "minmax"):
    """bf16 [N, K] -> (w_q uint32 [N, K/8], scales bf16 [N, K/64], biases bf16 [N, K/64]).

    ``variant="minmax"``: scale = (max - min)/15, bias = min per group;
    ``variant="zero_exact"``: the larger-magnitude edge is the bias and 0.0 is exactly
    representable.  Codes are rint((w - bias)/scale) clipped to 0..15.
    """
    _check_qparams(group_size, bits)
    _require_cuda("w", w, (torch.bfloat16,))
    if w.dim() != 2:
        raise ValueError("w must be 2-D [N, K]")
    if variant not in _VARIANTS:
        raise ValueError(f"variant must be one of {sorted(_VARIANTS)}")
    N, K = w.shape
    if K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    w = w.contiguous()
    wq = torch.empty((N, K * bits // 32), dtype=torch.uint32, device=w.device)
    s = torch.empty((N, K // group_size), dtype=torch.bfloat16, device=w.device)
    b = torch.empty_like(s)
    check(lib().qvx_quantize(_ptr(w), _ptr(wq), _ptr(s), _ptr(b), N, K, group_size, bits, _VARIANTS[variant],
                             _stream(w)), "qvx_quantize")
    return wq, s, b


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4) -> torch.Tensor:
    """bf16 [N, K] = scales * q + biases (mx.dequantize)."""
    _check_qparams(group_size, bits)
    w = _packed(w)
    _require_cuda("scales", scales, (torch.bfloat16,))
    _require_cuda("biases", biases, (torch.bfloat16,))
    N, KW = w.shape
    K = KW * 32 // bits
    if tuple(scales.shape) != (N, K // group_size) or tuple(biases.shape) != (N, K // group_size):
        raise ValueError("scales/biases shape does not match w")
    out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
    check(lib().qvx_dequantize(_ptr(w), _ptr(scales.contiguous()), _ptr(biases.contiguous()), _ptr(out), N, K,
                               group_size, bits, _stream(w)), "qvx_dequantize")
    return out


def dequantize_rows(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, ids: torch.Tensor,
                    group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """dequantize(w[ids], scales[ids], biases[ids]) without materialising the gather."""
    _check_qparams(group_size, bits)
    w = _packed(w)
    N, KW = w.shape
    K = KW * 32 // bits
    _require_cuda("ids", ids, (torch.int32, torch.int64))
    flat = ids.reshape(-1).to(torch.int32).contiguous()
    out = torch.empty((*ids.shape, K), dtype=torch.bfloat16, device=w.device)
    if flat.numel() == 0:
        return out
    check(lib().qvx_dequantize_rows(_ptr(w), _ptr(scales.contiguous()), _ptr(biases.contiguous()), _ptr(flat),
                                    flat.numel(), _ptr(out), N, K, group_size, bits, _stream(w)),
          "qvx_dequantize_rows")
    return out


_PROLOGUES = {"plain": _lib.QVX_IN_PLAIN, "rms_norm": _lib.QVX_IN_RMS_NORM, "swiglu": _lib.QVX_IN_SWIGLU,
              "gated_rms_norm": _lib.QVX_IN_GATED_RMS_NORM}
_EPILOGUES = {"plain": _lib.QVX_OUT_PLAIN, "swiglu_pairs": _lib.QVX_OUT_SWIGLU_PAIRS}


def _rows(t: torch.Tensor, name: str) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t
    if t2.stride(-1) != 1:
        raise ValueError(f"{name} must have unit stride along its rows")
    return t2


def qmv_fused(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
              prologue: str = "plain", norm_w: torch.Tensor | None = None, z: torch.Tensor | None = None,
              head_dim: int = 0, eps: float = 1e-6, resid: torch.Tensor | None = None,
              out: torch.Tensor | None = None, gather=None, group_size: int = 64, bits: int = 4,
              epilogue: str = "plain") -> torch.Tensor:
    """Decode projection (M <= 8 token rows) with a fused prologue and residual epilogue
    (qvx_qmv_fused):  y = resid + (prologue(x) @ dequant(w)^T)  (resid optional), where the
    prologue is "plain", "rms_norm" (norm_w [K]), "swiglu" (x = gate|up rows of 2K) or
    "gated_rms_norm" (per head of head_dim, norm_w [head_dim], z rows).  epilogue
    "swiglu_pairs": the weight rows are (gate, up) pairs and y [M, N/2] = silu(g) * u.
    ``gather`` is a qvx_gather descriptor (ctypes) for the sharded forms.  Returns y
    ([M, N], or [M, N/2]; ``out``)."""
    _check_qparams(group_size, bits)
    if prologue not in _PROLOGUES:
        raise ValueError(f"prologue must be one of {sorted(_PROLOGUES)}")
    _require_cuda("x", x, (torch.bfloat16,))
    w = _packed(w)
    N, KW = w.shape
    K = KW * 32 // bits
    x2 = _rows(x, "x")
    M = x2.shape[0]
    io = _lib.QvxQmvIO()
    io.prologue = _PROLOGUES[prologue]
    io.x_stride = x2.stride(0)
    io.eps = float(eps)
    if norm_w is not None:
        io.norm_w = norm_w.data_ptr()
    if z is not None:
        z2 = _rows(z, "z")
        io.z, io.z_stride = z2.data_ptr(), z2.stride(0)
    io.head_dim = int(head_dim)
    if resid is not None:
        r2 = _rows(resid, "resid")
        if tuple(r2.shape) != (M, N) or not r2.is_contiguous():
            raise ValueError("resid must be a contiguous [M, N] bf16 tensor")
        io.resid = r2.data_ptr()
    if epilogue not in _EPILOGUES:
        raise ValueError(f"epilogue must be one of {sorted(_EPILOGUES)}")
    io.epilogue = _EPILOGUES[epilogue]
    if out is None and not (gather is not None and gather.mode == _lib.QVX_EXCHANGE_GATHER):
        out = torch.empty((M, N // 2 if epilogue == "swiglu_pairs" else N), dtype=torch.bfloat16, device=x.device)
    import ctypes
    check(lib().qvx_qmv_fused(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), M, N, K, group_size, bits,
                              ctypes.byref(io), ctypes.byref(gather) if gather is not None else None, _stream(x2)),
          "qvx_qmv_fused")
    return out
