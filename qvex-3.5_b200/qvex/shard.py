"""Column sharding of quantized projections across GPUs, with an all-gather of the outputs.

Output rows (N) of a 4-bit g64 linear are independent and groups run along K, so rank r
of P owns the contiguous rows [r*N/P, (r+1)*N/P) of w, scales and biases and computes
y[:, shard] with the local kernel; an all-gather over NCCL (NVLink / NVSwitch) rebuilds
y.  Fused projections are sharded per component (``shard_fused``) so that a
nonlinearity that pairs components -- SwiGLU over gate|up, the DeltaNet split of
qkv|z|b|a -- finds both halves of its inputs on the same rank.

The pieces are separate so the host logic runs on CPU process groups (gloo) in tests:
``shard_rows`` / ``shard_linear`` / ``shard_fused`` only slice, ``gather_columns`` only
moves data, ``ShardedQLinear`` composes them with the CUDA kernel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .model import QLinear


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's rows; every rank gets the same count (n % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n % world:
        raise ValueError(f"{n} rows do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_linear(lin: QLinear, world: int, rank: int) -> QLinear:
    a, b = shard_rows(lin.w.shape[0], world, rank)
    return QLinear(lin.w[a:b].contiguous(), lin.scales[a:b].contiguous(), lin.biases[a:b].contiguous(),
                   lin.group_size, lin.bits)


def shard_fused(parts: list[QLinear], world: int, rank: int) -> QLinear:
    """Shard each component separately, then fuse the local pieces: the local output is
    [part0_shard | part1_shard | ...], so element-wise pairings of components stay local."""
    return QLinear.fuse([shard_linear(p, world, rank) for p in parts])


def gather_columns(local_y: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather row shards: local_y [..., N/P] on every rank -> y [..., N] (rank-major).

    For a single token the gathered buffer already is y; for M > 1 the [P, M, N/P] result
    is transposed into [M, P * N/P].
    """
    world = dist.get_world_size(group)
    lead = local_y.shape[:-1]
    n_loc = local_y.shape[-1]
    flat = local_y.reshape(-1, n_loc).contiguous()
    M = flat.shape[0]
    buf = torch.empty((world * M, n_loc), dtype=local_y.dtype, device=local_y.device)
    dist.all_gather_into_tensor(buf, flat, group=group)  # rank-major concat along dim 0
    buf = buf.view(world, M, n_loc)
    if M == 1:
        y = buf.view(1, world * n_loc)
    else:
        y = buf.permute(1, 0, 2).reshape(M, world * n_loc)
    if out is not None:
        out.view(M, world * n_loc).copy_(y)
        return out
    return y.reshape(*lead, world * n_loc)


class ShardedQLinear:
    """A QLinear whose output rows are spread over the ranks of ``group``."""

    def __init__(self, full: QLinear | list[QLinear], group=None, rank: int | None = None,
                 world: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if world is None else world
        self.rank = dist.get_rank(group) if rank is None else rank
        parts = full if isinstance(full, list) else [full]
        self.local = shard_fused(parts, self.world, self.rank)
        self.out_features = sum(p.w.shape[0] for p in parts)

    def __call__(self, x: torch.Tensor, *, gather: bool = True) -> torch.Tensor:
        y = self.local(x)
        return gather_columns(y, self.group) if gather and self.world > 1 else y
