"""Column sharding of quantized projections across GPUs, with an all-gather of the outputs.

Output rows (N) of a 4-bit g64 linear are independent and groups run along K, so rank r
of P owns the contiguous rows [r*N/P, (r+1)*N/P) of w, scales and biases and computes
y[:, shard] with the local kernel; an all-gather over NCCL (NVLink / NVSwitch) rebuilds
y.  Fused projections are sharded per component (``shard_fused``) so that a
nonlinearity that pairs components -- SwiGLU over gate|up, the DeltaNet split of
qkv|z|b|a -- finds both halves of its inputs on the same rank.

For decode (M <= 8) the all-gather can instead be fused into the projection kernel
(``qvx_qmv_allgather``): every rank stores its rows straight into every peer's receive
area (inbox) over NVLink as words that carry their launch's tag, and takes the peers'
rows out of its own inbox, so one kernel per projection does the compute and the
exchange, with no fence, signal or NCCL call.  ``PeerGather`` sets up those buffers: one
device allocation per rank, mapped into every rank's process with CUDA IPC.

The pieces are separate so the host logic runs on CPU process groups (gloo) in tests:
``shard_rows`` / ``shard_linear`` / ``shard_fused`` only slice, ``gather_columns`` only
moves data, ``plan_gather_layout`` / ``gather_descriptor`` only compute offsets and
addresses, ``ShardedQLinear`` composes them with the CUDA kernels.
"""
from __future__ import annotations

import ctypes

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


def part_order(sizes: list[int], world: int, device=None) -> torch.Tensor:
    """Column permutation from the rank-major order of a gathered fused projection (rank r's
    block holds its shard of every part, in part order) to the order of the unsharded fused
    projection (part j whole, then part j + 1): result[t] = gathered column of column t."""
    per = [shard_rows(n, world, 0)[1] for n in sizes]
    n_loc = sum(per)
    idx = []
    for j, pj in enumerate(per):
        off = sum(per[:j])
        for r in range(world):
            idx.extend(range(r * n_loc + off, r * n_loc + off + pj))
    return torch.tensor(idx, dtype=torch.long, device=device)


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


GATHER_ALIGN = 256
GATHER_M_MAX = 8  # tokens a fused decode projection gathers (qvx_qmv's M <= 8)


def plan_layout(sizes: list[tuple[int, int]]) -> tuple[list[int], list[int], int]:
    """Byte layout of one rank's PeerGather buffer from (output bytes, inbox bytes) per slot:
    the output and then the inbox, each 256-byte aligned.  Returns the outputs' offsets, the
    inboxes' offsets and the total size."""
    if any(o <= 0 or i <= 0 for o, i in sizes):
        raise ValueError("every region needs a positive size")

    def up(v):
        return (v + GATHER_ALIGN - 1) // GATHER_ALIGN * GATHER_ALIGN

    at = 0
    outs, inboxes = [], []
    for o, i in sizes:
        outs.append(at)
        at = up(at + o)
        inboxes.append(at)
        at = up(at + i)
    return outs, inboxes, at


def plan_gather_layout(region_bytes: list[int]) -> tuple[list[int], list[int], int]:
    """Layout of gather slots only: per slot the full output (``region_bytes`` of bf16) and
    its inbox, four times that (one 64-bit word, two outputs and a tag, per output pair, in
    two halves that alternating launches use)."""
    return plan_layout([(b, 4 * b) for b in region_bytes])


def reduce_slot_bytes(m_max: int, n: int, world: int) -> tuple[int, int]:
    """(partial-sum bytes, inbox bytes) of a row-parallel reduce slot: fp32 partials [m_max, n];
    an inbox of 64-bit (fp32, tag) words [2 halves][world][m_max][n]."""
    return 4 * m_max * n, 2 * world * m_max * n * 8


def gather_descriptor(bases: list[int], out_offset: int, inbox_offset: int, epoch_ptr: int, rank: int,
                      slot: int, n_total: int, row0: int):
    """qvx_gather for one projection: out[r] and inbox[r] = rank r's buffer + the slot's
    output and inbox offsets; epoch = this rank's counters (two words per slot, indexed by
    slot in the kernel)."""
    from . import _lib
    d = _lib.QvxGather()
    for r, base in enumerate(bases):
        d.out[r] = base + out_offset
        d.inbox[r] = base + inbox_offset
    d.epoch = epoch_ptr
    d.world, d.rank, d.n_total, d.row0, d.slot = len(bases), rank, n_total, row0, slot
    return d


def _ck(res):
    """Unwrap a cuda-python (error, value...) result, raising on an error."""
    err, *vals = res if isinstance(res, tuple) else (res,)
    if int(err) != 0:
        raise RuntimeError(f"CUDA runtime call failed: {err}")
    return vals[0] if len(vals) == 1 else (tuple(vals) if vals else None)


class _DeviceArray:
    """__cuda_array_interface__ over a raw device pointer (torch.as_tensor wraps it)."""

    def __init__(self, ptr: int, shape: tuple[int, ...]):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """Output regions and inboxes of fused column-sharded projections, one device
    buffer per rank of ``group`` mapped into every rank's process (CUDA IPC; peer access
    over NVLink).  ``region_bytes[i]`` is the size of slot i's full output; every rank must
    construct it with the same list, and keep it alive while its projections are in use.
    Set-up allocates and exchanges handles; the projections themselves allocate nothing."""

    def __init__(self, region_bytes: list[int], group=None, reduce: list[tuple[int, int]] | None = None):
        """``region_bytes``: one bf16 output size per gather slot; ``reduce``: (m_max, n) per
        row-parallel reduce slot (numbered after the gather slots)."""
        from cuda.bindings import runtime as rt
        from . import _lib
        self._rt = rt
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.QVX_MAX_RANKS:
            raise ValueError(f"{self.world} ranks; the fused gather supports up to {_lib.QVX_MAX_RANKS}")
        self.device = torch.cuda.current_device()
        _ck(rt.cudaSetDevice(self.device))
        reduce = list(reduce or [])
        self.reduce_shapes = reduce
        self.n_gather = len(region_bytes)
        sizes = [(b, 4 * b) for b in region_bytes] + [reduce_slot_bytes(m, n, self.world) for m, n in reduce]
        self.offsets, self.inboxes, self.nbytes = plan_layout(sizes)
        self.slots = len(sizes)
        self._next_reduce = self.n_gather
        self._own = _ck(rt.cudaMalloc(self.nbytes))
        _ck(rt.cudaMemset(self._own, 0, self.nbytes))
        _ck(rt.cudaDeviceSynchronize())
        handle = _ck(rt.cudaIpcGetMemHandle(self._own))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.reserved), group=group)
        self.base = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.base.append(int(self._own))
            else:
                h = rt.cudaIpcMemHandle_t()
                h.reserved = hb
                self.base.append(int(_ck(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess))))
        self.epoch = torch.zeros(2 * max(1, self.slots), dtype=torch.int32, device=self.device)
        self._next = 0
        dist.barrier(group)  # every rank has mapped every buffer before anyone stores

    def reserve(self) -> int:
        """Hands out the next gather slot."""
        if self._next >= self.n_gather:
            raise ValueError(f"all {self.n_gather} gather slots are taken")
        self._next += 1
        return self._next - 1

    def reserve_reduce(self) -> int:
        """Hands out the next reduce slot."""
        if self._next_reduce >= self.slots:
            raise ValueError(f"all {self.slots - self.n_gather} reduce slots are taken")
        self._next_reduce += 1
        return self._next_reduce - 1

    def reduce_descriptor(self, slot: int, n: int):
        """qvx_gather (mode QVX_EXCHANGE_REDUCE) of a reduce slot: out[rank] = this rank's fp32
        partial sums, inbox[r] = rank r's receive area, n_total = n, row0 = 0."""
        from . import _lib
        m_max, n_max = self.reduce_shapes[slot - self.n_gather]
        if n > n_max:
            raise ValueError(f"reduce slot {slot} holds {n_max} rows, not {n}")
        d = gather_descriptor(self.base, self.offsets[slot], self.inboxes[slot], self.epoch.data_ptr(), self.rank,
                              slot, n, 0)
        d.mode = _lib.QVX_EXCHANGE_REDUCE
        return d

    def descriptor(self, slot: int, n_total: int, row0: int):
        return gather_descriptor(self.base, self.offsets[slot], self.inboxes[slot], self.epoch.data_ptr(),
                                 self.rank, slot, n_total, row0)

    def output(self, slot: int, M: int, n_total: int) -> torch.Tensor:
        """This rank's full output of ``slot`` as a bf16 [M, n_total] tensor (a view of the
        shared buffer: the next call of that projection overwrites it)."""
        arr = _DeviceArray(self.base[self.rank] + self.offsets[slot], (M, n_total))
        return torch.as_tensor(arr, device=f"cuda:{self.device}").view(torch.bfloat16)

    def reset(self) -> None:
        """Puts every slot back in its starting state: zero inboxes and launch counters on every
        rank.  The ranks' counters of a slot stay in step only while every rank makes every
        call, so after a call that failed, timed out (QvexTimeout, device status
        QVX_ERR_TIMEOUT) or was skipped on any rank, every rank calls this before the next
        gathered projection.  Collective: all ranks of the group must call it."""
        rt = self._rt
        _ck(rt.cudaDeviceSynchronize())
        dist.barrier(self.group)   # no rank still stores into another's inbox
        _ck(rt.cudaMemset(self._own, 0, self.nbytes))
        self.epoch.zero_()
        _ck(rt.cudaDeviceSynchronize())
        dist.barrier(self.group)   # no rank starts a call while another still clears

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a device sync and a
        barrier, so no rank still stores into it)."""
        if self._own is None:
            return
        rt = self._rt
        _ck(rt.cudaDeviceSynchronize())
        dist.barrier(self.group)
        for r, p in enumerate(self.base):
            if r != self.rank:
                _ck(rt.cudaIpcCloseMemHandle(p))
        dist.barrier(self.group)
        _ck(rt.cudaFree(self._own))
        self._own = None


def qmv_allgather(local: QLinear, x: torch.Tensor, desc) -> None:
    """One fused launch: this rank's rows of ``local`` times x [M <= 8, K], stored into every
    rank's output region of ``desc`` (a PeerGather descriptor) through the inboxes."""
    from . import _lib
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("x must be a bf16 CUDA tensor")
    x = x.contiguous()
    M, K = x.shape
    w, s, b = local.w, local.scales, local.biases
    P = ctypes.c_void_p
    rc = _lib.lib().qvx_qmv_allgather(P(x.data_ptr()), P(w.data_ptr()), P(s.data_ptr()), P(b.data_ptr()),
                                      ctypes.byref(desc), M, w.shape[0], K, local.group_size, local.bits,
                                      P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "qvx_qmv_allgather")


class ShardedQLinear:
    """A QLinear whose output rows are spread over the ranks of ``group``.

    With ``peer`` (a PeerGather) decode calls (M <= 8) run the fused kernel: compute and
    all-gather in one launch, returning a view of the gathered output.  Otherwise, and for
    M > 8, the local kernel is followed by an NCCL all-gather."""

    def __init__(self, full: QLinear | list[QLinear], group=None, rank: int | None = None,
                 world: int | None = None, peer: PeerGather | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if world is None else world
        self.rank = dist.get_rank(group) if rank is None else rank
        parts = full if isinstance(full, list) else [full]
        self.local = shard_fused(parts, self.world, self.rank)
        self.out_features = sum(p.w.shape[0] for p in parts)
        self.peer = peer
        # Gathered rank by rank, the columns of a fused projection come out as
        # [rank 0: part 0 shard, part 1 shard, ...][rank 1: ...]; _perm puts them back in the
        # order of the unsharded QLinear.fuse(parts): [part 0][part 1]...
        self._perm = part_order(
            [p.w.shape[0] for p in parts], self.world, self.local.w.device) if len(parts) > 1 else None
        if peer is not None:
            n_loc = self.local.w.shape[0]
            if n_loc % 2:
                raise ValueError(f"the fused gather moves rows in pairs: {n_loc} rows per rank is odd "
                                 "(use the NCCL gather, peer=None)")
            self.slot = peer.reserve()
            self._desc = peer.descriptor(self.slot, self.out_features, self.rank * n_loc)

    def __call__(self, x: torch.Tensor, *, gather: bool = True) -> torch.Tensor:
        """y = x @ W^T: all columns in the unsharded order (gather=True), or only this rank's
        shard [part 0 shard | part 1 shard | ...] (gather=False)."""
        x2 = x.reshape(-1, x.shape[-1])
        if self.peer is not None and gather and x2.shape[0] <= GATHER_M_MAX:
            qmv_allgather(self.local, x2, self._desc)
            y = self.peer.output(self.slot, x2.shape[0], self.out_features)
            return self.in_part_order(y).reshape(*x.shape[:-1], self.out_features)
        y = self.local(x)
        return self.gather(y) if gather else y

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """NCCL all-gather of this rank's shard outputs, in the unsharded column order."""
        y = gather_columns(y_local, self.group) if self.world > 1 else y_local
        return self.in_part_order(y)

    def in_part_order(self, y: torch.Tensor) -> torch.Tensor:
        return y if self._perm is None else y.index_select(-1, self._perm)
