"""The reference's hot-path building blocks (engine/model.py) on libqvex.

``QLinear`` (engine/model.py:80-104), ``QEmbedding`` (:121-130) and ``RecurrentCache``
(:179-193) keep their constructor arguments, attributes and methods, so code written
against the reference's classes runs unchanged with torch CUDA tensors.
"""
from __future__ import annotations

import torch

from .core import QMM_MIN_M_PREPARED, dequantize_rows, qmm_prepare, quantized_matmul


class QLinear:
    """A projection whose weight is kept in the 4-bit affine group format; calling it
    returns x times the transposed dequantised weight, computed by libqvex."""

    def __init__(self, w, scales, biases, group_size=64, bits=4):
        self.w, self.scales, self.biases = w, scales, biases
        self.group_size, self.bits = group_size, bits
        self._prep = None  # the tensor-core path's weight prepass, made on first use

    @property
    def out_features(self) -> int:
        return self.w.shape[0]

    @property
    def in_features(self) -> int:
        return self.w.shape[1] * 32 // self.bits

    def prepared(self):
        """The weight prepass of the tensor-core path (qmm_prepare), made on the first call
        with QMM_MIN_M_PREPARED rows or more outside a CUDA-graph capture and kept (the
        weight is constant); None before that.  With it, calls of that many rows or more
        take the tensor-core path."""
        if self._prep is None and not torch.cuda.is_current_stream_capturing():
            self._prep = qmm_prepare(self.scales, self.biases, self.group_size, self.bits)
        return self._prep

    def __call__(self, x, *, out=None, workspace=None):
        prep = None
        if x.numel() >= QMM_MIN_M_PREPARED * self.in_features:
            prep = self.prepared()
        return quantized_matmul(x, self.w, self.scales, self.biases, transpose=True,
                                group_size=self.group_size, bits=self.bits, out=out, workspace=workspace,
                                prep=prep)

    @staticmethod
    def fuse(layers: list["QLinear"]) -> "QLinear":
        """One layer whose output rows are those of ``layers`` in order, for projections that
        read the same input: one launch then computes all of them, with identical results."""
        l0 = layers[0]
        if not all((l.group_size, l.bits) == (l0.group_size, l0.bits) for l in layers):
            raise AssertionError("fused layers must share the quantization (bits, group size)")
        return QLinear(
            torch.cat([l.w for l in layers]),
            torch.cat([l.scales for l in layers]),
            torch.cat([l.biases for l in layers]),
            l0.group_size, l0.bits,
        )


    @staticmethod
    def interleave(a: "QLinear", b: "QLinear") -> "QLinear":
        """One layer whose output rows alternate between ``a`` and ``b`` (a_0, b_0, a_1, b_1,
        ...): an MLP's gate|up with SwiGLU applied to adjacent row pairs (qvx_qmv_fused's
        swiglu_pairs epilogue, qvx_swiglu_pairs)."""
        if a.w.shape != b.w.shape or (a.group_size, a.bits) != (b.group_size, b.bits):
            raise AssertionError("interleaved layers must share the shape and the quantization")

        def mix(x, y):
            return torch.stack([x, y], dim=1).reshape(2 * x.shape[0], *x.shape[1:]).contiguous()

        return QLinear(mix(a.w, b.w), mix(a.scales, b.scales), mix(a.biases, b.biases), a.group_size, a.bits)


class QEmbedding:
    def __init__(self, w, scales, biases, group_size=64, bits=4):
        self.w, self.scales, self.biases = w, scales, biases
        self.group_size, self.bits = group_size, bits

    def __call__(self, ids):
        return dequantize_rows(self.w, self.scales, self.biases, ids, group_size=self.group_size, bits=self.bits)


class RecurrentCache:
    """Per-layer decode state of a gated-DeltaNet layer (convolution window and recurrent
    matrix) plus the copies needed to undo the newest token."""

    def __init__(self):
        self.conv = None   # [B, K-1, conv_dim]
        self.ssm = None    # [B, Hv, Dv, Dk] float32
        self.offset = 0
        self.conv_prev = self.ssm_prev = None  # states before the newest token, for a rejected draft

    def state(self):
        return [x for x in (self.conv, self.ssm) if x is not None]

    def rollback(self, n=1):
        if not (n == 1 and self.ssm_prev is not None):
            raise AssertionError("rollback restores one token, and only once after a keep_prev step")
        self.conv, self.ssm = self.conv_prev, self.ssm_prev
        self.conv_prev = self.ssm_prev = None
        self.offset -= 1
