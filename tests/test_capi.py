"""libqvex.so: it builds, loads, exports every entry point of include/qvex.h, and rejects
bad arguments before touching a GPU.  CPU only (no compute calls)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qvex.h"


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(qvx_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    from qvex import _lib
    from qvex.build import build
    build()
    return _lib.lib()


def test_every_header_symbol_is_exported(L):
    names = header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n


def test_binding_table_covers_header():
    from qvex import _lib
    assert sorted(_lib.SIGNATURES) == header_functions()


def test_version(L):
    assert L.qvx_version() >= 100


P = ctypes.c_void_p
DUMMY = P(4096)  # an aligned non-null address: never dereferenced, validation fails first


@pytest.mark.parametrize("M,N,K,gs,bits,code", [
    (0, 8, 64, 64, 4, 1),      # M < 1
    (9, 8, 64, 64, 4, 1),      # qmv is M <= 8
    (1, 8, 100, 64, 4, 1),     # K % 64
    (1, 0, 64, 64, 4, 1),      # N < 1
    (1, 8, 64, 32, 4, 2),      # group size not implemented
    (1, 8, 64, 64, 3, 2),      # 3-bit not implemented
])
def test_qmv_rejects_bad_arguments(L, M, N, K, gs, bits, code):
    rc = L.qvx_qmv(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, M, N, K, gs, bits, None)
    assert rc == code
    assert L.qvx_last_error()


def test_qmv_rejects_misaligned_x(L):
    assert L.qvx_qmv(P(4098), DUMMY, DUMMY, DUMMY, DUMMY, 1, 8, 64, 64, 4, None) == 3


def test_qmm_workspace_checks(L):
    # K = 64 is one stage, so there is no K split and the size asked for is the minimum
    need = L.qvx_qmm_workspace_size(64, 128, 64)
    assert need >= 64 * 64 * 2
    assert L.qvx_qmm(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 64, 128, 64, 64, 4, None, 0, None) == 6
    assert L.qvx_qmm(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 64, 128, 64, 64, 4, DUMMY, need - 1, None) == 6
    assert L.qvx_qmm(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 64, 128, 64, 64, 4, P(4096 + 16), need, None) == 3
    # K = 256 at one tile splits K, and the size includes the fp32 partial sums; a workspace
    # without them is accepted (the call runs unsplit), one without the rest is not
    split = L.qvx_qmm_workspace_size(64, 128, 256)
    assert split >= L.qvx_qmm_workspace_size(64, 128, 64) + 64 * 128 * 4
    assert L.qvx_qmm(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 64, 128, 256, 64, 4, DUMMY, split - 1, None) != 6
    assert L.qvx_qmm(DUMMY, DUMMY, DUMMY, DUMMY, DUMMY, 64, 128, 256, 64, 4, DUMMY, 1024, None) == 6


def test_qmm_prepare_checks(L):
    """The weight prepass buffer: its size (per-row exponents, then per-group multipliers at
    a 256-byte boundary), and the argument checks of qvx_qmm_prepare / qvx_qmm_prepared."""
    need = L.qvx_qmm_prepared_bytes(300, 4096)
    assert need >= 300 * 4 + 300 * 64 * 8
    assert L.qvx_qmm_prepared_bytes(0, 4096) == 0 and L.qvx_qmm_prepared_bytes(8, 100) == 0
    assert L.qvx_qmm_prepare(DUMMY, DUMMY, 300, 4096, 64, 4, None, need, None) == 1       # null prep
    assert L.qvx_qmm_prepare(DUMMY, DUMMY, 300, 4096, 32, 4, DUMMY, need, None) == 2      # group size
    assert L.qvx_qmm_prepare(DUMMY, DUMMY, 300, 4096, 64, 4, P(4096 + 16), need, None) == 3  # alignment
    assert L.qvx_qmm_prepare(DUMMY, DUMMY, 300, 4096, 64, 4, DUMMY, need - 1, None) == 6  # too small
    assert L.qvx_qmm_prepared(DUMMY, DUMMY, DUMMY, DUMMY, 64, 300, 4096, 64, 4, None, 0, None) == 6
    assert L.qvx_qmm_prepared(DUMMY, DUMMY, P(4096 + 16), DUMMY, 64, 300, 4096, 64, 4, DUMMY, 1 << 30, None) == 3


def test_gated_delta_rejects_bad_shapes(L):
    args = [DUMMY] * 11
    assert L.qvx_gated_delta(*args, 1, 1, 3, 32, 128, 128, None) == 1    # Hv % Hk
    assert L.qvx_gated_delta(*args, 1, 1, 16, 32, 96, 128, None) == 2    # Dk not 32/64/128
    assert L.qvx_gated_delta(*args, 1, 0, 16, 32, 128, 128, None) == 1   # T < 1
    assert L.qvx_gated_delta(*args, 1, 1, 16, 32, 128, 120, None) == 1   # Dv % 16


def test_quantize_rejects(L):
    assert L.qvx_quantize(DUMMY, DUMMY, DUMMY, DUMMY, 4, 100, 64, 4, 0, None) == 1
    assert L.qvx_quantize(DUMMY, DUMMY, DUMMY, DUMMY, 4, 128, 64, 4, 7, None) == 1
    assert L.qvx_quantize(DUMMY, DUMMY, DUMMY, DUMMY, 4, 128, 128, 4, 0, None) == 2


def test_python_front_end_rejects_cpu_tensors():
    import torch
    import qvex
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    w = torch.zeros(8, 8, dtype=torch.int32)
    s = torch.zeros(8, 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        qvex.quantized_matmul(x, w, s, s)
    with pytest.raises(NotImplementedError):
        qvex.quantized_matmul(x, w, s, s, bits=3)
    with pytest.raises(NotImplementedError):
        qvex.quantized_matmul(x, w, s, s, transpose=False)


def test_qlinear_fuse_and_rollback_host_logic():
    import torch
    from qvex import QLinear, RecurrentCache
    a = QLinear(torch.zeros(4, 8, dtype=torch.int32), torch.zeros(4, 1), torch.ones(4, 1), 64, 4)
    b = QLinear(torch.ones(2, 8, dtype=torch.int32), torch.ones(2, 1), torch.zeros(2, 1), 64, 4)
    f = QLinear.fuse([a, b])
    assert f.w.shape == (6, 8) and f.out_features == 6 and f.in_features == 64
    assert torch.equal(f.w[4:], b.w)
    with pytest.raises(AssertionError):
        QLinear.fuse([a, QLinear(b.w, b.scales, b.biases, 32, 4)])
    c = RecurrentCache()
    with pytest.raises(AssertionError):
        c.rollback(1)
    c.ssm, c.conv, c.offset = "s1", "c1", 5
    c.ssm_prev, c.conv_prev = "s0", "c0"
    c.rollback(1)
    assert (c.ssm, c.conv, c.offset, c.ssm_prev) == ("s0", "c0", 4, None)


def test_qmv_allgather_rejects_bad_descriptors(L):
    from qvex import _lib
    g = _lib.QvxGather()
    for r in range(2):
        g.out[r] = 4096
        g.inbox[r] = 4096
    g.epoch = 4096
    g.world, g.rank, g.n_total, g.row0, g.slot = 2, 0, 16, 0, 0

    def call(gg, M=1, N=8):
        return L.qvx_qmv_allgather(DUMMY, DUMMY, DUMMY, DUMMY, ctypes.byref(gg) if gg else None,
                                   M, N, 512, 64, 4, None)
    assert call(None) == 1
    g.world = 9
    assert call(g) == 1            # more ranks than QVX_MAX_RANKS
    g.world, g.rank = 2, 2
    assert call(g) == 1            # rank outside the world
    g.rank = 1
    g.row0 = 12
    assert call(g) == 1            # rows past n_total
    g.row0 = 4
    assert call(g) == 1            # shards not in rank order
    g.row0 = 8
    assert call(g, N=6) == 1       # shards not equal (2 x 6 != 16)
    g.n_total = 14
    assert call(g, N=7) == 1       # odd row count: rows move in pairs
    g.n_total = 16
    g.inbox[0] = None
    assert call(g) == 1            # a peer's inbox missing
    g.inbox[0] = 4100
    assert call(g) == 1            # an inbox not 8-byte aligned
    g.inbox[0] = 4096
    assert call(g, M=9) == 1       # decode only
    assert ctypes.sizeof(_lib.QvxGather) == 160  # 8 + 8 pointers, epoch, 5 ints (+4 padding)


def test_sampler_rejects(L):
    F = ctypes.c_float
    # M, V, dtype
    assert L.qvx_sample_scores(DUMMY, 2, None, DUMMY, 1, 100, F(0.6), F(0.95), 20, F(0), None) == 1
    assert L.qvx_sample_scores(DUMMY, 0, None, DUMMY, 1, 0, F(0.6), F(0.95), 20, F(0), None) == 1
    assert L.qvx_sample_scores(None, 0, None, DUMMY, 1, 100, F(0.6), F(0.95), 20, F(0), None) == 1
    assert L.qvx_sample_scores(P(4097), 1, None, DUMMY, 1, 100, F(0.6), F(0.95), 20, F(0), None) == 3
    # top_k beyond the supported candidate count, and top_p over the whole vocabulary
    assert L.qvx_sample_scores(DUMMY, 0, None, DUMMY, 1, 5000, F(0.6), F(0.95), 2000, F(0), None) == 2
    assert L.qvx_sample_scores(DUMMY, 0, None, DUMMY, 1, 5000, F(0.6), F(0.95), 0, F(0), None) == 2
    assert L.qvx_sample_scores(DUMMY, 0, None, DUMMY, 0, 5000, F(0.6), F(0.95), 20, F(0), None) == 0
    assert L.qvx_sample_pick(None, DUMMY, 1, 100, 1, 0, 0, None) == 1
    assert L.qvx_sample_pick(DUMMY, DUMMY, 1, 0, 1, 0, 0, None) == 1


def test_qk_condition_rejects(L):
    assert L.qvx_qk_condition(DUMMY, DUMMY, DUMMY, DUMMY, 8, 127, None) == 1   # odd D
    assert L.qvx_qk_condition(DUMMY, DUMMY, DUMMY, DUMMY, 8, 258, None) == 1   # D > 256
    assert L.qvx_qk_condition(DUMMY, DUMMY, DUMMY, DUMMY, -1, 128, None) == 1
    assert L.qvx_qk_condition(P(4098), DUMMY, DUMMY, DUMMY, 8, 128, None) == 3
    assert L.qvx_qk_condition(None, None, None, None, 0, 128, None) == 0       # nothing to do


def test_attention_split_count_host_logic():
    """Decode attention's key ranges per KV head: one CTA per SM over all (sequence, KV
    head) pairs, at most 64, and no more than one range per 128 cache positions."""
    from qvex.glue import split_count
    assert split_count(1, 8, 148) == 18
    assert split_count(1, 8, 148, cap=4352) == 18
    assert split_count(1, 8, 148, cap=1280) == 10
    assert split_count(1, 8, 148, cap=100) == 1
    assert split_count(64, 8, 148, cap=4096) == 1
    assert split_count(1, 1, 148) == 64
    assert split_count(4, 2, 148, cap=300) == 3
