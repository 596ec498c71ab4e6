"""qvex: B200-native (sm_100a) quantized linear + gated-DeltaNet hot path of QVex.

Public surface (mirrors the reference's):
  quantized_matmul, quantize, dequantize   -- mx.quantized_matmul / mx.quantize / mx.dequantize
  gated_delta, qmv_multi, qk_condition     -- engine/kernels.py, engine/model.py:275-277
  QLinear, QEmbedding, RecurrentCache      -- engine/model.py
  Sampler, SamplingParams                  -- engine/sampler.py (scores, pick) on the GPU
  shard                                    -- column sharding over GPUs with an all-gather
All compute runs in libqvex.so (C ABI, include/qvex.h) through ctypes.
"""
from .core import dequantize, dequantize_rows, qmm_workspace_size, quantize, quantized_matmul
from .kernels import gated_delta, qk_condition, qmv_multi
from .model import QEmbedding, QLinear, RecurrentCache
from .sampler import Sampler, SamplingParams, sample_pick, sample_scores
from ._lib import QvexError, QvexTimeout, lib as _load_lib

__all__ = [
    "quantized_matmul", "quantize", "dequantize", "dequantize_rows", "qmm_workspace_size",
    "gated_delta", "qk_condition", "qmv_multi", "QLinear", "QEmbedding", "RecurrentCache", "QvexError", "QvexTimeout",
    "Sampler", "SamplingParams", "sample_scores", "sample_pick", "load_library",
]


def load_library():
    """Load libqvex.so now (raises if it is not built)."""
    return _load_lib()
