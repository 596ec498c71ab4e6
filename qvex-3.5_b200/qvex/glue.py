"""The layer glue of a Qwen3.5 decoder layer on libqvex, with MLX-style functional calls.

``rms_norm`` (mx.fast.rms_norm, engine/model.py:314,316,335; with the residual add of
:315-316 in front), ``gated_rms_norm`` (_gated_rmsnorm, :138-143), ``swiglu`` (_swiglu,
:133-135), ``deltanet_conv`` (GatedDeltaNet.__call__ from the in_proj split to the
gated_delta call, :259-277), ``deltanet_decode`` (conv, recurrence and gated norm in one
kernel for up to 4 tokens) and ``attention`` (Attention.__call__ between the projections,
:213-232, with KVCache.update, :156-170).  Every call runs one libqvex entry point on the
current CUDA stream; there is no other path.
"""
from __future__ import annotations

import math

import torch

from ._lib import _P, check, lib
from .core import _ptr, _require_cuda, _stream


def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float, *, resid: torch.Tensor | None = None,
             out: torch.Tensor | None = None, h_out: torch.Tensor | None = None):
    """rms_norm(x [+ resid]) * w over the last axis.  With ``resid`` returns (out, h) where
    h = x + resid (written into ``h_out`` if given, which may be ``x`` or ``resid``)."""
    _require_cuda("x", x, (torch.bfloat16,))
    D = x.shape[-1]
    x = x.contiguous()
    if resid is not None:
        _require_cuda("resid", resid, (torch.bfloat16,))
        if resid.shape != x.shape:
            raise ValueError("resid must have x's shape")
        resid = resid.contiguous()
        if h_out is None:
            h_out = torch.empty_like(x)
    if out is None:
        out = torch.empty_like(x)
    if w is not None:
        _require_cuda("w", w, (torch.bfloat16,))
        if w.numel() != D:
            raise ValueError(f"w has {w.numel()} elements for rows of {D}")
    check(lib().qvx_rms_norm(_ptr(x), _ptr(resid), _ptr(w), float(eps), _ptr(h_out), _ptr(out), x.numel() // D, D,
                             _stream(x)), "qvx_rms_norm")
    return (out, h_out) if resid is not None else out


def add(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(a + b) elementwise (same shapes, contiguous); ``out`` may be a or b."""
    _require_cuda("a", a, (torch.bfloat16,))
    _require_cuda("b", b, (torch.bfloat16,))
    if a.shape != b.shape or not a.is_contiguous() or not b.is_contiguous():
        raise ValueError("add needs two contiguous tensors of one shape")
    if out is None:
        out = torch.empty_like(a)
    check(lib().qvx_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(a)), "qvx_add")
    return out


def gated_rms_norm(y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, *,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """y [T, H, D] (any leading shape flattened to T), z [T, >= H*D] (row stride = z.stride(0),
    unit stride along the row), w [D] -> bf16 [T, H*D]."""
    _require_cuda("y", y, (torch.bfloat16,))
    _require_cuda("z", z, (torch.bfloat16,))
    _require_cuda("w", w, (torch.bfloat16,))
    D = w.numel()
    z2 = z if z.dim() == 2 else z.reshape(-1, z.shape[-1])
    if z2.stride(-1) != 1:
        raise ValueError("z must have unit stride along its rows")
    T = z2.shape[0]
    y2 = y.contiguous()
    if y2.numel() % (T * D):
        raise ValueError(f"y has {y2.numel()} elements, not a multiple of {T} tokens x {D}")
    H = y2.numel() // (T * D)
    if out is None:
        out = torch.empty((T, H * D), dtype=torch.bfloat16, device=y.device)
    check(lib().qvx_gated_rms_norm(_ptr(y2), _ptr(z2), z2.stride(0), _ptr(w.contiguous()), float(eps), _ptr(out), T,
                                   H, D, _stream(y)), "qvx_gated_rms_norm")
    return out


def swiglu(gu: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """gu [M, 2I] = [gate | up] (row stride gu.stride(0)) -> bf16 [M, I]."""
    _require_cuda("gu", gu, (torch.bfloat16,))
    g2 = gu.reshape(-1, gu.shape[-1]) if gu.dim() != 2 else gu
    if g2.stride(-1) != 1:
        raise ValueError("gu must have unit stride along its rows")
    M, I2 = g2.shape
    if out is None:
        out = torch.empty((*gu.shape[:-1], I2 // 2), dtype=torch.bfloat16, device=gu.device)
    check(lib().qvx_swiglu(_ptr(g2), g2.stride(0), _ptr(out), M, I2 // 2, _stream(gu)), "qvx_swiglu")
    return out


def swiglu_pairs(gu: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """gu [M, 2I] = (g_0, u_0, g_1, u_1, ...) (row stride gu.stride(0)) -> bf16 [M, I]:
    SwiGLU of an MLP whose gate|up weight rows are interleaved in pairs."""
    _require_cuda("gu", gu, (torch.bfloat16,))
    g2 = gu.reshape(-1, gu.shape[-1]) if gu.dim() != 2 else gu
    if g2.stride(-1) != 1:
        raise ValueError("gu must have unit stride along its rows")
    M, I2 = g2.shape
    if out is None:
        out = torch.empty((*gu.shape[:-1], I2 // 2), dtype=torch.bfloat16, device=gu.device)
    check(lib().qvx_swiglu_pairs(_ptr(g2), g2.stride(0), _ptr(out), M, I2 // 2, _stream(gu)), "qvx_swiglu_pairs")
    return out


def deltanet_conv(proj: torch.Tensor, conv_w: torch.Tensor, state: torch.Tensor, Hk: int, Hv: int, Dk: int, Dv: int,
                  *, state_out: torch.Tensor | None = None, keep_mid: bool = False, outs=None):
    """proj [B, T, >= qkv|z|b|a] (in_proj output), conv_w fp32 [C, 4], state bf16 [B, 3, C].
    Returns (q, k, v, a, b, state_out[, state_mid]); q/k [B, T, Hk, Dk], v [B, T, Hv, Dv],
    a/b [B, T, Hv].  ``state_out`` may be ``state`` (in place) when T <= 64."""
    _require_cuda("proj", proj, (torch.bfloat16,))
    _require_cuda("state", state, (torch.bfloat16,))
    _require_cuda("conv_w", conv_w, (torch.float32,))
    B, T, S = proj.shape
    if proj.stride(-1) != 1 or proj.stride(0) != T * proj.stride(1):
        raise ValueError("proj rows must be evenly strided with unit stride along a row")
    C, KW = conv_w.shape
    dev = proj.device
    if outs is None:
        outs = (torch.empty((B, T, Hk, Dk), dtype=torch.bfloat16, device=dev),
                torch.empty((B, T, Hk, Dk), dtype=torch.bfloat16, device=dev),
                torch.empty((B, T, Hv, Dv), dtype=torch.bfloat16, device=dev),
                torch.empty((B, T, Hv), dtype=torch.bfloat16, device=dev),
                torch.empty((B, T, Hv), dtype=torch.bfloat16, device=dev))
    q, k, v, a, b = outs
    if state_out is None:
        state_out = torch.empty_like(state)
    mid = torch.empty_like(state) if keep_mid else None
    check(lib().qvx_deltanet_conv(_ptr(proj), proj.stride(1), _ptr(conv_w.contiguous()), KW, _ptr(state.contiguous()),
                                  _ptr(state_out), _ptr(mid), _ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), B, T, Hk, Hv,
                                  Dk, Dv, _stream(proj)), "qvx_deltanet_conv")
    return (q, k, v, a, b, state_out, mid) if keep_mid else (q, k, v, a, b, state_out)


def deltanet_decode_supported(T: int, Hk: int, Hv: int, Dk: int, Dv: int) -> bool:
    """Whether qvx_deltanet_decode takes this shape (else run the three kernels)."""
    return 1 <= T <= 4 and Dk in (64, 128) and Hv % Hk == 0 and Dv % 32 == 0 and (Hv // Hk) * (Dv // 32) == 8


def deltanet_decode_preferred(B: int, T: int, Hk: int, Hv: int, Dk: int, Dv: int, device=None) -> bool:
    """Whether to run the fused kernel: a supported shape whose B * Hk clusters of 8 CTAs
    are resident at once (at most one per SM).  Measured on B200 at Qwen3.5-9B shapes: at
    batch 1 (16 clusters) the fused kernel saves ~3 us per layer; at batch 64 (1024
    clusters, several waves of a latency-bound kernel) it is far slower than the three
    kernels, whose grids spread over the whole GPU."""
    if not deltanet_decode_supported(T, Hk, Hv, Dk, Dv):
        return False
    return B * Hk <= torch.cuda.get_device_properties(device).multi_processor_count


def deltanet_decode(proj: torch.Tensor, conv_w: torch.Tensor, conv_state: torch.Tensor, A_log: torch.Tensor,
                    dt_bias: torch.Tensor, state: torch.Tensor, norm_w: torch.Tensor, eps: float, Hk: int, Hv: int,
                    Dk: int, Dv: int, *, conv_out: torch.Tensor | None = None, state_out: torch.Tensor | None = None,
                    keep_mid: bool = False, out: torch.Tensor | None = None):
    """GatedDeltaNet from the in_proj output to the out_proj input in one kernel (T <= 4).
    Returns (out [B, T, Hv*Dv], conv_out, state_out[, conv_mid, state_mid]); conv_out and
    state_out may be the input buffers (in place)."""
    _require_cuda("proj", proj, (torch.bfloat16,))
    _require_cuda("conv_state", conv_state, (torch.bfloat16,))
    _require_cuda("state", state, (torch.float32,))
    B, T, S = proj.shape
    if proj.stride(-1) != 1 or proj.stride(0) != T * proj.stride(1):
        raise ValueError("proj rows must be evenly strided with unit stride along a row")
    C, KW = conv_w.shape
    dev = proj.device
    if out is None:
        out = torch.empty((B, T, Hv * Dv), dtype=torch.bfloat16, device=dev)
    if conv_out is None:
        conv_out = torch.empty_like(conv_state)
    if state_out is None:
        state_out = torch.empty_like(state)
    cmid = torch.empty_like(conv_state) if keep_mid else None
    smid = torch.empty_like(state) if keep_mid else None
    check(lib().qvx_deltanet_decode(_ptr(proj), proj.stride(1), _ptr(conv_w.contiguous()), KW, _ptr(conv_state),
                                    _ptr(conv_out), _ptr(cmid), _ptr(A_log), _ptr(dt_bias), _ptr(state), _ptr(state_out),
                                    _ptr(smid), _ptr(norm_w), float(eps), _ptr(out), B, T, Hk, Hv, Dk, Dv,
                                    _stream(proj)), "qvx_deltanet_decode")
    return (out, conv_out, state_out, cmid, smid) if keep_mid else (out, conv_out, state_out)


def rope_inv_freq(rotary_dim: int, base: float, device) -> torch.Tensor:
    """fp32 rope frequencies base^(-2i/rotary_dim), computed in double, rounded once."""
    i = torch.arange(rotary_dim // 2, dtype=torch.float64)
    return (base ** (-2.0 * i / rotary_dim)).to(torch.float32).to(device)


def attention_workspace(B: int, Hkv: int, G: int, L: int, D: int, nsplit: int, device) -> torch.Tensor | None:
    """Zeroed workspace for the split-key decode form, or None when it does not apply."""
    n = int(lib().qvx_attention_workspace_size(B, Hkv, G, L, D, nsplit))
    return torch.zeros(n, dtype=torch.uint8, device=device) if n else None


def split_count(B: int, Hkv: int, sms: int, cap: int | None = None) -> int:
    """Key ranges per KV head for decode: one CTA per SM at most over all (sequence, KV head)
    pairs (a CTA of 8 warps, each warp streaming rounds of 8 keys), at most 64, and with a
    cache of ``cap`` positions no more than one range per 128 of them.  Measured on B200
    (batch 1, 8 KV heads): 1024 positions 12.1 us at 9 ranges against 14.2 at 18; 4096
    positions 17.9 us at 18 against 20.2 at 12."""
    n = max(1, min(64, sms // max(1, B * Hkv)))
    if cap is not None:
        n = min(n, max(1, -(-int(cap) // 128)))
    return n


def default_splits(B: int, Hkv: int, device=None, cap: int | None = None) -> int:
    """split_count on ``device`` (the current CUDA device by default)."""
    return split_count(B, Hkv, torch.cuda.get_device_properties(device).multi_processor_count, cap)


def attention(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, eps: float, inv_freq: torch.Tensor,
              k_cache: torch.Tensor, v_cache: torch.Tensor, pos, H: int, Hkv: int, D: int, *, scale: float | None = None,
              workspace: torch.Tensor | None = None, nsplit: int = 0, out: torch.Tensor | None = None,
              q_buf: torch.Tensor | None = None) -> torch.Tensor:
    """qkv [B, L, >= (2H + 2Hkv) D] -> bf16 [B, L, H*D]; writes the new keys and values into
    the caches [B, Hkv, cap, D] at positions [pos, pos + L).  ``pos`` is an int or a device
    int32 tensor of one element (then read on the device at run time)."""
    _require_cuda("qkv", qkv, (torch.bfloat16,))
    B, L, S = qkv.shape
    if qkv.stride(-1) != 1 or qkv.stride(0) != L * qkv.stride(1):
        raise ValueError("qkv rows must be evenly strided with unit stride along a row")
    cap = k_cache.shape[2]
    rd = 2 * inv_freq.numel()
    dev = qkv.device
    if out is None:
        out = torch.empty((B, L, H * D), dtype=torch.bfloat16, device=dev)
    if q_buf is None:
        q_buf = torch.empty((B, L, H, D), dtype=torch.bfloat16, device=dev)
    pos_dev = pos if torch.is_tensor(pos) else None
    pos_host = 0 if torch.is_tensor(pos) else int(pos)
    ws_bytes = 0 if workspace is None else workspace.numel()
    check(lib().qvx_attention(_ptr(qkv), qkv.stride(1), _ptr(q_norm), _ptr(k_norm), float(eps), _ptr(inv_freq), rd,
                              _ptr(k_cache), _ptr(v_cache), cap, _ptr(pos_dev), pos_host, _ptr(q_buf), _ptr(out), B, L,
                              H, Hkv, D, float(D ** -0.5 if scale is None else scale), _ptr(workspace), ws_bytes,
                              int(nsplit), _stream(qkv)), "qvx_attention")
    return out
