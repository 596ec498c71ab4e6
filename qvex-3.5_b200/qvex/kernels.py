"""The reference's custom kernels (engine/kernels.py) with the same call surface.

``gated_delta`` keeps the argument list, shapes and return tuple of
engine/kernels.py:92-116; ``qmv_multi`` keeps engine/kernels.py:197-211 (its K % 512
restriction is lifted: any K % 64 == 0 works).
"""
from __future__ import annotations

import torch

from ._lib import _P, check, lib
from .core import _ptr, _require_cuda, _stream, quantized_matmul


def gated_delta(q, k, v, a, b, A_log, dt_bias, state, keep_mid: bool = False, *, out_state=None):
    """
    q, k:  [B, T, Hk, Dk] bf16   v: [B, T, Hv, Dv] bf16   a, b: [B, T, Hv] bf16
    A_log, dt_bias: [Hv] (any float dtype; used as fp32)
    state: [B, Hv, Dv, Dk] float32
    returns y [B, T, Hv, Dv] (q.dtype), new state (+ state before the last step if keep_mid)

    ``out_state`` may be given to receive the new state (it may be ``state`` itself for an
    in-place update); by default a fresh tensor is returned, as in the reference.
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b)):
        _require_cuda(name, t, (torch.bfloat16,))
    _require_cuda("state", state, (torch.float32,))
    if k.dim() != 4 or q.shape != k.shape or v.dim() != 4:
        raise ValueError("q, k must be [B, T, Hk, Dk] and v [B, T, Hv, Dv]")
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2:]
    if tuple(v.shape[:2]) != (B, T) or tuple(a.shape) != (B, T, Hv) or tuple(b.shape) != (B, T, Hv):
        raise ValueError("v, a, b shapes do not match q/k")
    if tuple(state.shape) != (B, Hv, Dv, Dk):
        raise ValueError(f"state must be [{B}, {Hv}, {Dv}, {Dk}], got {tuple(state.shape)}")
    dev = q.device
    A_log = A_log.to(device=dev, dtype=torch.float32).contiguous()
    dt_bias = dt_bias.to(device=dev, dtype=torch.float32).contiguous()
    if A_log.numel() != Hv or dt_bias.numel() != Hv:
        raise ValueError("A_log and dt_bias must have Hv elements")
    q, k, v, a, b, state = (t.contiguous() for t in (q, k, v, a, b, state))
    y = torch.empty((B, T, Hv, Dv), dtype=q.dtype, device=dev)
    if out_state is None:
        out_state = torch.empty_like(state)
    elif out_state.shape != state.shape or out_state.dtype != torch.float32 or not out_state.is_contiguous():
        raise ValueError("out_state must be a contiguous float32 tensor shaped like state")
    mid = torch.empty_like(state) if keep_mid else None
    check(lib().qvx_gated_delta(_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(A_log), _ptr(dt_bias),
                                _ptr(state), _ptr(y), _ptr(out_state), _ptr(mid), B, T, Hk, Hv, Dk, Dv,
                                _stream(q)), "qvx_gated_delta")
    return (y, out_state, mid) if keep_mid else (y, out_state)


def qk_condition(q, k):
    """q, k [..., Dk] bf16 -> (Dk^-1 * rms_norm(q), Dk^-1/2 * rms_norm(k)), the conditioning
    GatedDeltaNet applies before gated_delta (engine/model.py:275-277).  New tensors."""
    _require_cuda("q", q, (torch.bfloat16,))
    _require_cuda("k", k, (torch.bfloat16,))
    if q.shape != k.shape:
        raise ValueError("q and k must have the same shape")
    D = q.shape[-1]
    q, k = q.contiguous(), k.contiguous()
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    check(lib().qvx_qk_condition(_ptr(q), _ptr(k), _ptr(qo), _ptr(ko), q.numel() // D, D, _stream(q)),
          "qvx_qk_condition")
    return qo, ko


def qmv_multi(x, w, scales, biases):
    """x [M, K] (M small), w [N, K/8] uint32 4-bit/group-64 -> y [M, N]"""
    if x.dim() != 2:
        raise ValueError("x must be [M, K]")
    if x.shape[0] > 8:
        raise ValueError("qmv_multi is the M <= 8 path")
    return quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4)
