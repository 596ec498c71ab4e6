"""Tensor-parallel Qwen3.5 over 1/2/4/8 GPUs: column-sharded projections paired with
row-parallel ones, so that each decoder layer exchanges twice per step instead of once per
projection.

Rank r of P holds (parameter names as in the reference's checkpoint, engine/model.py:342-397):
  * gated DeltaNet: key heads [r Hk/P, (r+1) Hk/P) and value heads [r Hv/P, (r+1) Hv/P) --
    their rows of in_proj_qkv (q, k and v parts), in_proj_z, in_proj_b, in_proj_a, their conv
    channels, A_log, dt_bias; the recurrence, conv window and gated norm of those heads stay
    local (grouped heads map inside a rank: value head h reads key head h / (Hv / Hk));
    out_proj keeps the matching K columns (row-parallel);
  * attention: query heads [r H/P, ...) and KV heads [r Hkv/P, ...) -- their rows of q_proj,
    k_proj, v_proj, their part of the KV cache; o_proj keeps the matching K columns;
  * MLP: rows [r I/P, (r+1) I/P) of gate_proj and up_proj (SwiGLU stays local), the same K
    columns of down_proj;
  * lm_head: vocabulary rows [r V/P, ...) (column-sharded, gathered); the embedding and the
    norm weights whole.
The residual stream is replicated.  The row-parallel projections' partial sums are summed
over the ranks: in decode (B <= 8 tokens) inside the projection kernel (qvx_qmv_fused with
QVX_EXCHANGE_REDUCE: fp32 partials exchanged between twin CTAs over NVLink, summed in rank
order, residual added), elsewhere by an NCCL all-reduce of the bf16 partials.  lm_head's
rows are gathered in its kernel (QVX_EXCHANGE_GATHER) or by NCCL.  Per decode step that is
2 exchanges per layer + 1: 65 for the 9B shape instead of one per projection (145).
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from .model import QLinear
from .shard import PeerGather, shard_rows


def rows_of(P: dict, name: str, ranges: list[tuple[int, int]]) -> None:
    """Keeps rows ``ranges`` (concatenated) of quantized module ``name`` in P (in place)."""
    for suffix in ("weight", "scales", "biases"):
        t = P[f"{name}.{suffix}"]
        P[f"{name}.{suffix}"] = torch.cat([t[a:b] for a, b in ranges]).contiguous()


def cols_of(P: dict, name: str, c0: int, c1: int, group_size: int = 64, bits: int = 4) -> None:
    """Keeps input columns [c0, c1) of quantized module ``name`` (whole groups)."""
    if c0 % group_size or c1 % group_size:
        raise ValueError(f"columns [{c0}, {c1}) do not fall on {group_size}-element groups")
    per_word = 32 // bits
    P[f"{name}.weight"] = P[f"{name}.weight"][:, c0 // per_word:c1 // per_word].contiguous()
    for suffix in ("scales", "biases"):
        P[f"{name}.{suffix}"] = P[f"{name}.{suffix}"][:, c0 // group_size:c1 // group_size].contiguous()


def shard_params(cfg, P: dict, world: int, rank: int):
    """(local config, local parameters) of rank ``rank`` of ``world`` from the full
    reference-named parameters (the dict is copied; tensors are sliced)."""
    H, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
    Dk, Dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
    I, V = cfg.intermediate_size, cfg.vocab_size
    for what, n in (("attention heads", H), ("KV heads", Hkv), ("DeltaNet key heads", Hk),
                    ("DeltaNet value heads", Hv), ("MLP rows", I), ("vocabulary rows", V)):
        if n % world:
            raise ValueError(f"{n} {what} do not split over {world} ranks")
    L = dict(P)
    hk0, hk1 = shard_rows(Hk, world, rank)
    hv0, hv1 = shard_rows(Hv, world, rank)
    h0, h1 = shard_rows(H, world, rank)
    g0, g1 = shard_rows(Hkv, world, rank)
    i0, i1 = shard_rows(I, world, rank)
    kd, vd = Hk * Dk, Hv * Dv
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}"
        m = f"{pre}.mlp"
        rows_of(L, f"{m}.gate_proj", [(i0, i1)])
        rows_of(L, f"{m}.up_proj", [(i0, i1)])
        cols_of(L, f"{m}.down_proj", i0, i1, *cfg.qparams(f"{m}.down_proj"))
        if cfg.is_linear(i):
            la = f"{pre}.linear_attn"
            qkv_rows = [(hk0 * Dk, hk1 * Dk), (kd + hk0 * Dk, kd + hk1 * Dk), (2 * kd + hv0 * Dv, 2 * kd + hv1 * Dv)]
            rows_of(L, f"{la}.in_proj_qkv", qkv_rows)
            rows_of(L, f"{la}.in_proj_z", [(hv0 * Dv, hv1 * Dv)])
            rows_of(L, f"{la}.in_proj_b", [(hv0, hv1)])
            rows_of(L, f"{la}.in_proj_a", [(hv0, hv1)])
            cw = L[f"{la}.conv1d.weight"]
            L[f"{la}.conv1d.weight"] = torch.cat([cw[a:b] for a, b in qkv_rows]).contiguous()
            L[f"{la}.A_log"] = L[f"{la}.A_log"][hv0:hv1].contiguous()
            L[f"{la}.dt_bias"] = L[f"{la}.dt_bias"][hv0:hv1].contiguous()
            cols_of(L, f"{la}.out_proj", hv0 * Dv, hv1 * Dv, *cfg.qparams(f"{la}.out_proj"))
        else:
            sa = f"{pre}.self_attn"
            rows_of(L, f"{sa}.q_proj", [(h0 * 2 * D, h1 * 2 * D)])
            rows_of(L, f"{sa}.k_proj", [(g0 * D, g1 * D)])
            rows_of(L, f"{sa}.v_proj", [(g0 * D, g1 * D)])
            cols_of(L, f"{sa}.o_proj", h0 * D, h1 * D, *cfg.qparams(f"{sa}.o_proj"))
    v0, v1 = shard_rows(V, world, rank)
    rows_of(L, "lm_head", [(v0, v1)])
    local = dataclasses.replace(cfg, num_attention_heads=H // world, num_key_value_heads=Hkv // world,
                                linear_num_key_heads=Hk // world, linear_num_value_heads=Hv // world,
                                intermediate_size=I // world)
    return local, L


@dataclasses.dataclass
class TP:
    """A rank's place in a tensor-parallel model: process group, and (for decode with the
    exchanges fused into the projections) the mapped peer buffers and per-layer slots."""
    group: object
    world: int
    rank: int
    vocab: int
    peer: PeerGather | None = None
    m_max: int = 8

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather_cols(self, y: torch.Tensor) -> torch.Tensor:
        from .shard import gather_columns
        return gather_columns(y, self.group) if self.world > 1 else y


def attach(model, tp: TP, fused_exchange: bool = True) -> None:
    """Makes ``model`` (built from shard_params output) tensor-parallel: eager forwards
    all-reduce the row-parallel projections' partial sums and all-gather lm_head's rows with
    NCCL; with ``fused_exchange`` a PeerGather is set up (collective) and graph decode of
    B <= 8 sequences exchanges inside the projection kernels."""
    model.tp = tp
    for layer in model.layers:
        layer.tp = tp
    H = model.cfg.hidden_size
    if not fused_exchange or tp.world == 1:
        return
    n_layers = len(model.layers)
    v_loc = model.lm_head.out_features
    tp.peer = PeerGather([tp.m_max * v_loc * tp.world * 2], group=tp.group,
                         reduce=[(tp.m_max, H)] * (2 * n_layers))
    for layer in model.layers:
        layer.tp_desc = (tp.peer.reduce_descriptor(tp.peer.reserve_reduce(), H),
                         tp.peer.reduce_descriptor(tp.peer.reserve_reduce(), H))
    slot = tp.peer.reserve()
    model.lm_slot = slot
    model.lm_desc = tp.peer.descriptor(slot, v_loc * tp.world, tp.rank * v_loc)


def close(model) -> None:
    tp = getattr(model, "tp", None)
    if tp is not None and tp.peer is not None:
        tp.peer.close()
        tp.peer = None
