"""Projection shapes of one decode step of a Qwen3.5-9B-shaped hybrid model.

Derived the way the reference builds its layers (engine/model.py): every 4th layer is
gated full attention (Config.is_linear, :73-74), the rest gated DeltaNet; DeltaNet's
qkv|z|b|a projections are fused into one in_proj (:244-251), MLP gate|up into one
gate_up (:296), attention q_proj emits query and gate (2 * heads * head_dim, :213-214).
The KV-head count is not fixed by the benchmark configuration; 8 is assumed and kept a
parameter.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Qwen35Shape:
    hidden: int = 4096
    intermediate: int = 12288
    layers: int = 32
    full_attention_interval: int = 4
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    lin_key_heads: int = 16
    lin_value_heads: int = 32
    lin_key_dim: int = 128
    lin_value_dim: int = 128
    vocab: int = 248320

    def is_linear(self, i: int) -> bool:
        return (i + 1) % self.full_attention_interval != 0

    def decode_linears(self) -> list[tuple[str, int, int]]:
        """(name, N, K) of every quantized linear, in execution order."""
        h = self.hidden
        key_dim = self.lin_key_heads * self.lin_key_dim
        value_dim = self.lin_value_heads * self.lin_value_dim
        conv_dim = 2 * key_dim + value_dim
        out = []
        for i in range(self.layers):
            if self.is_linear(i):
                out.append((f"layers.{i}.linear_attn.in_proj", conv_dim + value_dim + 2 * self.lin_value_heads, h))
                out.append((f"layers.{i}.linear_attn.out_proj", h, value_dim))
            else:
                out.append((f"layers.{i}.self_attn.q_proj", 2 * self.heads * self.head_dim, h))
                out.append((f"layers.{i}.self_attn.k_proj", self.kv_heads * self.head_dim, h))
                out.append((f"layers.{i}.self_attn.v_proj", self.kv_heads * self.head_dim, h))
                out.append((f"layers.{i}.self_attn.o_proj", h, self.heads * self.head_dim))
            out.append((f"layers.{i}.mlp.gate_up", 2 * self.intermediate, h))
            out.append((f"layers.{i}.mlp.down", h, self.intermediate))
        out.append(("lm_head", self.vocab, h))
        return out


def qlinear_bytes(N: int, K: int, group_size: int = 64, bits: int = 4) -> int:
    """Bytes of a 4-bit g64 linear: packed codes + bf16 scales and biases."""
    return N * K * bits // 8 + N * (K // group_size) * 2 * 2


def qmv_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic bytes of one qmv launch: weights once, x and y once."""
    return qlinear_bytes(N, K) + M * K * 2 + M * N * 2
