"""Multi-rank host logic of column sharding on CPU process groups (gloo, world size 2).

The CUDA kernel is replaced by a dense CPU matmul of the dequantised shard (computed with
the oracle), so what is tested here is the slicing, the all-gather layout and the
failure behaviour of the collective -- the same code the NCCL path runs.
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense(lin):
    """float32 [N, K] dequantised weight of a QLinear held as CPU tensors (oracle)."""
    import oracle as O
    w = lin.w.numpy().view(np.uint32)
    s = lin.scales.view(torch.int16).numpy().view(np.uint16)
    b = lin.biases.view(torch.int16).numpy().view(np.uint16)
    return torch.from_numpy(O.bf16_to_f32(O.dequantize(w, s, b)))


def _make_linear(N, K, seed):
    from make_golden import qmv_inputs
    from qvex.model import QLinear
    _, _, w, s, b = qmv_inputs(1, K, N, seed)
    return QLinear(torch.from_numpy(w.view(np.int32)), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
                   torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))


def _worker(rank, world, port, case, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    for p in (root / "qvex-3.5_b200", root / "oracle", root / "tests" / "golden"):
        sys.path.insert(0, str(p))
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        from qvex.shard import gather_columns, shard_fused, shard_linear, shard_rows
        if case == "gather":
            lin = _make_linear(48, 128, 1)
            full = _dense(lin)
            for M in (1, 3):
                x = torch.from_numpy(np.random.default_rng(M).standard_normal((M, 128)).astype(np.float32))
                loc = shard_linear(lin, world, rank)
                y_loc = x @ _dense(loc).T
                a, b = shard_rows(48, world, rank)
                assert torch.allclose(y_loc, (x @ full.T)[:, a:b])
                y = gather_columns(y_loc)
                assert y.shape == (M, 48)
                assert torch.allclose(y, x @ full.T, atol=1e-5)
        elif case == "fused":
            gate, up = _make_linear(32, 64, 2), _make_linear(32, 64, 3)
            loc = shard_fused([gate, up], world, rank)
            a, b = shard_rows(32, world, rank)
            dl = _dense(loc)
            assert torch.equal(dl[:16], _dense(gate)[a:b]) and torch.equal(dl[16:], _dense(up)[a:b])
        elif case == "fused_gather":
            # a gathered fused projection (parts of different sizes, as DeltaNet's
            # qkv|z|b|a) must come back in the column order of the unsharded fuse
            from qvex.model import QLinear
            from qvex.shard import ShardedQLinear
            parts = [_make_linear(n, 64, 10 + i) for i, n in enumerate((32, 16, 8))]
            fused = QLinear.fuse(parts)
            sl = ShardedQLinear(parts, rank=rank, world=world)
            x = torch.from_numpy(np.random.default_rng(5).standard_normal((3, 64)).astype(np.float32))
            y_loc = x @ _dense(sl.local).T
            y = sl.gather(y_loc)
            assert y.shape == (3, 56)
            assert torch.allclose(y, x @ _dense(fused).T, atol=1e-4)
        elif case == "rank_dies":
            if rank == 1:
                raise SystemExit(0)  # leaves between steps without joining the collective
            t0 = __import__("time").time()
            try:
                gather_columns(torch.zeros(1, 4))
                q.put((rank, "no error"))
                return
            except Exception:
                q.put((rank, f"raised after {__import__('time').time() - t0:.1f}s"))
                return
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized() and case != "rank_dies":
            dist.destroy_process_group()


def _run(case, world=2, expect=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    n_expected = world if expect is None else len(expect)
    for _ in range(n_expected):
        r, msg = q.get(timeout=120)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("case", ["gather", "fused", "fused_gather"])
def test_sharding_world2(case):
    res = _run(case)
    assert res == {0: "ok", 1: "ok"}, res


def test_rank_that_leaves_is_detected_by_collective_timeout():
    res = _run("rank_dies", expect=[0])
    assert res[0].startswith("raised"), res


def test_shard_rows_rules():
    from qvex.shard import shard_rows
    assert shard_rows(248320, 8, 7) == (217280, 248320)
    assert shard_rows(12352, 8, 0) == (0, 1544)
    with pytest.raises(ValueError):
        shard_rows(10, 4, 0)
    with pytest.raises(ValueError):
        shard_rows(8, 2, 2)


def test_plan_gather_layout():
    from qvex.shard import plan_gather_layout
    outs, inboxes, total = plan_gather_layout([2 * 1024, 300, 16])
    assert outs[0] == 0
    assert all(o % 256 == 0 for o in outs + inboxes)
    # each slot: its output, then an inbox four times its size (two halves of one 64-bit
    # word per output pair)
    assert inboxes[0] == 2048 and outs[1] == inboxes[0] + 8192
    assert inboxes[1] == outs[1] + 512 and outs[2] == inboxes[1] + 1280
    assert inboxes[2] == outs[2] + 256 and total == inboxes[2] + 256
    with pytest.raises(ValueError):
        plan_gather_layout([0])


def test_gather_descriptor_addresses():
    """Every rank's output and inbox of a slot sit at the same offsets of that rank's buffer;
    the descriptor carries them per rank, and the counters of this rank."""
    from qvex.shard import gather_descriptor, plan_gather_layout
    outs, inboxes, total = plan_gather_layout([2 * 4096] * 150)
    bases = [1 << 40, 2 << 40]
    for slot in (0, 97, 149):
        d = gather_descriptor(bases, outs[slot], inboxes[slot], 12345 << 8, 1, slot, 8192, 4096)
        assert [d.out[r] for r in range(2)] == [b + outs[slot] for b in bases]
        assert [d.inbox[r] for r in range(2)] == [b + inboxes[slot] for b in bases]
        assert d.epoch == 12345 << 8 and d.slot == slot and d.world == 2 and d.rank == 1
        # a slot's inbox lies between its output and the next slot's output
        nxt = outs[slot + 1] if slot + 1 < 150 else total
        assert outs[slot] + 2 * 4096 <= inboxes[slot] and inboxes[slot] + 4 * 2 * 4096 <= nxt




def test_sharded_qlinear_rejects_odd_rows_for_fused_gather():
    """The fused gather moves rows in pairs, so an odd per-rank row count is refused when
    the layer is built, before any slot is taken."""
    import torch
    from qvex.model import QLinear
    from qvex.shard import ShardedQLinear

    class Peer:
        taken = 0

        def reserve(self):
            Peer.taken += 1
            return 0

        def descriptor(self, *a):
            return None
    lin = QLinear(torch.zeros(6, 8, dtype=torch.int32), torch.zeros(6, 1, dtype=torch.bfloat16),
                  torch.zeros(6, 1, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="pairs"):
        ShardedQLinear(lin, rank=0, world=2, peer=Peer())
    assert Peer.taken == 0
    ok = ShardedQLinear(QLinear(torch.zeros(8, 8, dtype=torch.int32), torch.zeros(8, 1, dtype=torch.bfloat16),
                                torch.zeros(8, 1, dtype=torch.bfloat16)), rank=1, world=2, peer=Peer())
    assert ok.local.w.shape[0] == 4 and Peer.taken == 1


def test_part_order_permutation():
    """Rank-major gathered columns of a fused [a|b] projection map back to [a|b]."""
    from qvex.shard import part_order
    sizes, world = [8, 4], 2
    # gathered: rank 0 holds a[0:4], b[0:2]; rank 1 holds a[4:8], b[2:4]
    gathered = ["a0", "a1", "a2", "a3", "b0", "b1", "a4", "a5", "a6", "a7", "b2", "b3"]
    perm = part_order(sizes, world).tolist()
    assert [gathered[i] for i in perm] == [f"a{i}" for i in range(8)] + [f"b{i}" for i in range(4)]
    assert sorted(perm) == list(range(12))
