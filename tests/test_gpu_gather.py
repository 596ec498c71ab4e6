"""Fused column-sharded decode projection (qvx_qmv_allgather) on all visible GPUs.

One child process per GPU (2, 4 or 8 of them: the largest power of two the box has) sets
up a PeerGather (CUDA IPC mappings, exchanged over
a gloo process group: no NCCL) and run sharded projections; each rank's gathered output
must equal, bit for bit, the single-GPU qvx_qmv of the unsharded weights (a row's
arithmetic does not depend on how rows are split).  Covered: M = 1, 3 and 8, two calls in
a row with different inputs, the same projection launched twice back to back (the
second launch overlaps the first through programmatic dependent launch), one projection
called with a different token count in between (another grid, so another set of CTAs
writes each inbox word: the launch tags must still tell old words from new), slot
numbers above 120, a fused two-part projection (gathered columns in the unsharded
[gate | up] order), and PeerGather.reset() between calls.  Skipped with fewer than two
GPUs.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [(1, 4096, 1024), (3, 1024, 768), (8, 2048, 512)]  # M, K, N (N split over ranks)


def _child(rank, world, port, q):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    for p in (root / "qvex-3.5_b200", root / "oracle", root / "tests" / "golden"):
        sys.path.insert(0, str(p))
    try:
        import torch.distributed as dist
        import qvex
        from make_golden import qmv_inputs
        from qvex.model import QLinear
        from qvex.shard import PeerGather, ShardedQLinear
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        qvex.load_library()
        # 120 unused slots first: the projections below use high slot numbers, so a mistake in
        # the per-slot counters or region offsets lands in someone else's memory
        peer = PeerGather([256] * 120 + [8 * N * 2 for _, _, N in CASES] + [8 * 512 * 2])
        for _ in range(120):
            peer.reserve()
        ok = True
        msgs = []
        for M, K, N in CASES:
            x1, _, w, s, b = qmv_inputs(M, K, N, seed=500 + N)
            x2 = qmv_inputs(M, K, N, seed=900 + N)[0]
            x3 = qmv_inputs(4 if M == 1 else 1, K, N, seed=700 + N)[0]  # another token count

            def dev(a):
                return torch.from_numpy(np.ascontiguousarray(a)).cuda()
            full = QLinear(dev(w).view(torch.int32), dev(s).view(torch.bfloat16), dev(b).view(torch.bfloat16))
            lin = ShardedQLinear(full, rank=rank, world=world, peer=peer)
            for xa in (x1, x2, x2, x3, x1):
                xt = dev(xa).view(torch.bfloat16)
                y = lin(xt).clone()
                ref = full(xt)
                torch.cuda.synchronize()
                if not torch.equal(y.view(torch.int16), ref.view(torch.int16)):
                    ok = False
                    diff = (y.float() - ref.float()).abs().max().item()
                    msgs.append(f"rank {rank} M={M} K={K} N={N}: max diff {diff}")
            # the same slot twice back to back, then one check of the last result
            xt = dev(x1).view(torch.bfloat16)
            lin(xt)
            y = lin(xt).clone()
            torch.cuda.synchronize()
            if not torch.equal(y.view(torch.int16), full(xt).view(torch.int16)):
                ok = False
                msgs.append(f"rank {rank} M={M}: back-to-back launches differ")
        # a fused [gate | up] projection: the gathered columns come back in the unsharded order
        parts = []
        for i in range(2):
            _, _, w, s, b = qmv_inputs(1, 1024, 256, seed=40 + i)
            parts.append(QLinear(dev(w).view(torch.int32), dev(s).view(torch.bfloat16), dev(b).view(torch.bfloat16)))
        fused = QLinear.fuse(parts)
        lin = ShardedQLinear(parts, rank=rank, world=world, peer=peer)
        xt = dev(qmv_inputs(2, 1024, 8, seed=77)[0]).view(torch.bfloat16)
        for it in range(2):
            y = lin(xt).clone()
            torch.cuda.synchronize()
            if not torch.equal(y.view(torch.int16), fused(xt).view(torch.int16)):
                ok = False
                msgs.append(f"rank {rank}: fused two-part projection differs (call {it})")
            if it == 0:
                peer.reset()  # every slot back to zero on every rank; calls carry on from there
        status = qvex._lib.device_status(torch.cuda.current_stream().cuda_stream)
        if status:
            ok = False
            msgs.append(f"rank {rank}: device status {status}")
        peer.close()
        dist.destroy_process_group()
        q.put((rank, ok, msgs))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, [f"rank {rank}: {type(e).__name__}: {e}"]))


def _world():
    n = min(torch.cuda.device_count(), 8)
    return 8 if n >= 8 else 4 if n >= 4 else 2 if n >= 2 else 1


def test_fused_allgather_matches_single_gpu_qmv():
    world = _world()
    if world < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_child, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), [m for _, _, ms in results for m in ms]
