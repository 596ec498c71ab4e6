"""qvx_qmm_noalloc: the prefill quantized matmul for callers that cannot allocate device
memory (hosts that reach the library only through its C ABI with no device allocator,
engines whose memory pool forbids cudaMalloc while serving).  Its scratch is a 16 MiB
array built into the library instead of a caller workspace.

Checked here through the C ABI: two calls in a row, the second smaller and with an odd
number of quantisation groups so that it runs over what the first left in the shared
scratch, each against qvx_qmm with a freshly allocated workspace on the same inputs
(rel-L2 <= 1e-3, the matmul tolerance of the other parity tests).  This file is named to
be collected last; it needs nothing from the other test files.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from make_golden import qmv_inputs

MATMUL_TOL = 1e-3
SCRATCH_BYTES = 16 << 20
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def L():
    import qvex
    from qvex import _lib
    from qvex.build import build
    build()
    qvex.load_library()
    return _lib.lib()


def _rel_l2(a, b):
    a = O.bf16_to_f32(a).astype(np.float64)
    b = O.bf16_to_f32(b).astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _device(torch, a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.bfloat16)
    elif a.dtype == np.uint32:
        t = t.view(torch.int32)
    return t.cuda()


def _host(t):
    return t.view(__import__("torch").int16).cpu().numpy().view(np.uint16)


def _run(L, torch, inputs, allocating):
    """One call through the C ABI: qvx_qmm with a torch workspace, or qvx_qmm_noalloc."""
    from qvex import _lib
    x, w, s, b = (_device(torch, a) for a in inputs)
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    stream = P(torch.cuda.current_stream().cuda_stream)
    ptrs = [P(t.data_ptr()) for t in (x, w, s, b, y)]
    if allocating:
        need = L.qvx_qmm_workspace_size(M, N, K)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc = L.qvx_qmm(*ptrs, M, N, K, 64, 4, P(ws.data_ptr()), need, stream)
    else:
        rc = L.qvx_qmm_noalloc(*ptrs, M, N, K, 64, 4, stream)
    _lib.check(rc, "qmm")
    torch.cuda.synchronize()
    return _host(y)


@pytest.mark.gpu
def test_noalloc_matches_qvx_qmm_on_two_calls_in_a_row(L):
    import torch
    first = qmv_inputs(512, 2048, 4096, seed=9001)   # x, x_f32, w, scales, biases
    second = qmv_inputs(130, 1088, 1000, seed=9002)  # 17 groups: a zero-padded last stage
    first, second = [(z[0], z[2], z[3], z[4]) for z in (first, second)]
    y1 = _run(L, torch, first, allocating=False)
    y2 = _run(L, torch, second, allocating=False)
    assert _rel_l2(y1, _run(L, torch, first, allocating=True)) <= MATMUL_TOL
    assert _rel_l2(y2, _run(L, torch, second, allocating=True)) <= MATMUL_TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(L):
    """Rejected before any GPU work, so this runs without a GPU too."""
    M, N, K = 4096, 12288, 4096
    assert L.qvx_qmm_workspace_size(M, N, K) > SCRATCH_BYTES
    dummy = P(4096)
    rc = L.qvx_qmm_noalloc(dummy, dummy, dummy, dummy, dummy, M, N, K, 64, 4, None)
    assert rc == 6  # QVX_ERR_WORKSPACE
    assert b"16777216" in L.qvx_last_error()
    assert L.qvx_qmm_workspace_size(1024, 12288, 4096) <= SCRATCH_BYTES
