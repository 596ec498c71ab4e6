"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and the golden
fixtures made from the reference's own code.

Tolerances: bit-exact for codes, packed words, bf16 scales/biases and dequantised
values; bf16 matmul outputs rel-L2 <= 1e-3 against the oracle's bf16 output;
gated-DeltaNet y (bf16) rel-L2 <= 1e-3 and fp32 states rel-L2 <= 1e-4.
"""
import numpy as np
import pytest
import torch

import detrand
import oracle as O
from make_golden import gd_inputs, qmv_inputs

pytestmark = pytest.mark.gpu

MATMUL_TOL = 1e-3
STATE_TOL = 1e-4


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.bfloat16)
    elif a.dtype == np.uint32:
        t = t.view(torch.int32)
    return t.cuda()


def host_u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def rel_l2(a, b):
    a = O.bf16_to_f32(a).astype(np.float64) if a.dtype == np.uint16 else a.astype(np.float64)
    b = O.bf16_to_f32(b).astype(np.float64) if b.dtype == np.uint16 else b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def qvex():
    import qvex as q
    from qvex.build import build
    build()
    q.load_library()
    return q


# ------------------------------------------------------------------ qmv (M <= 8)

@pytest.mark.parametrize("name", sorted(p.name for p in __import__("conftest").GOLDEN.glob("qmv_*.npz")))
def test_qmv_matches_reference_kernel_fixture(qvex, golden_dir, name):
    z = np.load(golden_dir / name)
    y = qvex.quantized_matmul(dev(z["x"]), dev(z["w"]), dev(z["scales"]), dev(z["biases"]))
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y), z["y"]) <= MATMUL_TOL


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("N,K", [(12288, 4096), (4096, 12288), (67, 64), (1, 128), (1000, 2048), (33, 16384)])
def test_qmv_matches_oracle(qvex, M, N, K):
    x, _, w, s, b = qmv_inputs(M, K, N, seed=M * 1000 + N + K)
    ref = O.qmm_exact(x, w, s, b)
    y = qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b))
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y), ref) <= MATMUL_TOL


@pytest.mark.parametrize("M", [1, 2, 3, 8])
def test_qmv_wide_dynamic_range(qvex, M):
    """x spanning twelve decades inside each 32-input slice: the fixed-point planes are
    scaled to the slice max, so small inputs lose bits, but the error stays a fraction of
    the slice max and y stays within tolerance (M >= 3 uses 14-bit planes)."""
    N, K = 1000, 4096
    x, _, w, s, b = qmv_inputs(M, K, N, seed=4242 + M)
    mag = 10.0 ** (detrand.uniform((M, K), 77 + M) * 12.0 - 6.0)
    x = O.f32_to_bf16(O.bf16_to_f32(x) * mag.astype(np.float32))
    ref = O.qmm_exact(x, w, s, b)
    y = qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b))
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y), ref) <= MATMUL_TOL


def test_qmv_quantized_from_real_weights(qvex):
    # config-2 style weights (N(0, 0.02) quantized), M = 2 verify shape
    w = O.f32_to_bf16(detrand.normal((512, 4096), 21) * 0.02)
    wq, s, b = O.quantize(w, 64, "minmax")
    x = O.f32_to_bf16(detrand.normal((2, 4096), 22))
    ref = O.qmm_exact(x, wq, s, b)
    y = qvex.quantized_matmul(dev(x), dev(wq), dev(s), dev(b))
    assert rel_l2(host_u16(y), ref) <= MATMUL_TOL


def test_qmv_leading_dims_and_out(qvex):
    x, _, w, s, b = qmv_inputs(4, 1024, 96, seed=5)
    ref = O.qmm_exact(x, w, s, b)
    out = torch.empty(2, 2, 96, dtype=torch.bfloat16, device="cuda")
    y = qvex.quantized_matmul(dev(x).view(2, 2, 1024), dev(w), dev(s), dev(b), out=out)
    assert y.data_ptr() == out.data_ptr()
    assert rel_l2(host_u16(y.reshape(4, 96)), ref) <= MATMUL_TOL


def test_qmv_multi_alias_and_qlinear(qvex):
    x, _, w, s, b = qmv_inputs(2, 4096, 300, seed=8)
    ref = O.qmm_exact(x, w, s, b)
    y1 = qvex.qmv_multi(dev(x), dev(w), dev(s), dev(b))
    lin = qvex.QLinear(dev(w), dev(s), dev(b), 64, 4)
    y2 = lin(dev(x))
    assert torch.equal(y1, y2)
    assert rel_l2(host_u16(y1), ref) <= MATMUL_TOL


def test_qlinear_fuse_equals_separate(qvex):
    parts = [qmv_inputs(1, 1024, n, seed=40 + n) for n in (96, 32, 8)]
    x = dev(parts[0][0])
    lins = [qvex.QLinear(dev(p[2]), dev(p[3]), dev(p[4])) for p in parts]
    fused = qvex.QLinear.fuse(lins)
    y = fused(x)
    sep = torch.cat([l(x) for l in lins], dim=-1)
    assert torch.equal(y, sep)


# ------------------------------------------------------------------ quantize / dequantize

@pytest.mark.parametrize("variant", ["minmax", "zero_exact"])
def test_quantize_bit_exact_config2(qvex, variant):
    w = O.f32_to_bf16(detrand.normal((12288, 4096), 2) * 0.02)
    wq_r, s_r, b_r = O.quantize(w, 64, variant)
    wq, s, b = qvex.quantize(dev(w), 64, 4, variant=variant)
    torch.cuda.synchronize()
    assert np.array_equal(wq.view(torch.int32).cpu().numpy().view(np.uint32), wq_r)
    assert np.array_equal(host_u16(s), s_r)
    assert np.array_equal(host_u16(b), b_r)


@pytest.mark.parametrize("variant", ["minmax", "zero_exact"])
def test_quantize_edge_cases_bit_exact(qvex, variant):
    w = (detrand.normal((8, 256), 3) * 0.02).astype(np.float32)
    w[0] = 0.0
    w[1] = 3.0
    w[2, :64] = 1e30
    w[3, :64] = -1e-38
    w[4, ::2] = 65504.0
    w[5] = np.linspace(-1, 1, 256)
    w[6, :64] = 7.0
    w[6, 1] = -7.0
    wb = O.f32_to_bf16(w)
    wq_r, s_r, b_r = O.quantize(wb, 64, variant)
    wq, s, b = qvex.quantize(dev(wb), 64, 4, variant=variant)
    assert np.array_equal(wq.view(torch.int32).cpu().numpy().view(np.uint32), wq_r)
    assert np.array_equal(host_u16(s), s_r)
    assert np.array_equal(host_u16(b), b_r)


@pytest.mark.parametrize("variant", ["minmax", "zero_exact"])
def test_quantize_nonfinite_bit_exact(qvex, variant):
    """NaN and infinite elements: NaN codes clamp to 0, an infinite edge makes the scale
    infinite; the fast no-clamp path must hand every such group to the exact path."""
    w = (detrand.normal((6, 256), 5) * 0.02).astype(np.float32)
    w[0, 5] = np.nan
    w[0, 70] = np.nan
    w[0, 71] = np.nan
    w[1, 3] = np.inf
    w[2, 64] = -np.inf
    w[3, :64] = np.nan
    w[4, 128:192] = np.nan
    w[4, 130] = 1.0
    w[5, ::3] = np.nan
    wb = O.f32_to_bf16(w)
    wq_r, s_r, b_r = O.quantize(wb, 64, variant)
    wq, s, b = qvex.quantize(dev(wb), 64, 4, variant=variant)
    assert np.array_equal(wq.view(torch.int32).cpu().numpy().view(np.uint32), wq_r)
    assert np.array_equal(host_u16(s), s_r)
    assert np.array_equal(host_u16(b), b_r)


@pytest.mark.parametrize("N,K", [(1000, 4160), (3, 64), (777, 1024), (4099, 576)])
def test_quantize_ragged_shapes_bit_exact(qvex, N, K):
    """Group counts that leave a partial last stage (512 groups per stage), one group per
    row, and more stages than SMs with a ragged tail."""
    w = O.f32_to_bf16(detrand.normal((N, K), N + K) * 0.05)
    wq_r, s_r, b_r = O.quantize(w, 64, "minmax")
    wq, s, b = qvex.quantize(dev(w), 64, 4)
    torch.cuda.synchronize()
    assert np.array_equal(wq.view(torch.int32).cpu().numpy().view(np.uint32), wq_r)
    assert np.array_equal(host_u16(s), s_r)
    assert np.array_equal(host_u16(b), b_r)


def test_pack_order_on_device(qvex, golden_dir):
    # quantize a row whose codes are known, compare the packed words with the reference pack
    z = np.load(golden_dir / "pack_4bit.npz")
    codes = z["codes"][3:4, :64]                     # 0..15, 0..15, ...
    w = O.f32_to_bf16(codes.astype(np.float32))     # scale 1, bias 0 under minmax
    wq, s, b = qvex.quantize(dev(w), 64, 4)
    assert np.array_equal(wq.view(torch.int32).cpu().numpy().view(np.uint32), z["packed"][3:4, :8])


def test_dequantize_bit_exact(qvex):
    x, _, w, s, b = qmv_inputs(1, 4096, 2048, seed=77)
    ref = O.dequantize(w, s, b)
    out = qvex.dequantize(dev(w), dev(s), dev(b))
    assert np.array_equal(host_u16(out), ref)


def test_dequantize_rows_gather(qvex):
    _, _, w, s, b = qmv_inputs(1, 512, 100, seed=78)
    ids = np.array([[5, 0, 99], [42, 42, 7]], np.int32)
    full = O.dequantize(w, s, b)
    emb = qvex.QEmbedding(dev(w), dev(s), dev(b))
    out = emb(torch.from_numpy(ids).cuda())
    assert out.shape == (2, 3, 512)
    assert np.array_equal(host_u16(out).reshape(6, 512), full[ids.reshape(-1)])


def test_dequantize_rows_bad_id_sets_device_status(qvex):
    from qvex import _lib
    _, _, w, s, b = qmv_inputs(1, 128, 10, seed=79)
    _lib.device_status(torch.cuda.current_stream().cuda_stream)  # clear
    out = qvex.dequantize_rows(dev(w), dev(s), dev(b), torch.tensor([1, 10], dtype=torch.int32, device="cuda"))
    st = _lib.device_status(torch.cuda.current_stream().cuda_stream)
    assert st == _lib.QVX_ERR_INVALID
    assert torch.all(out[1] == 0)
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


# ------------------------------------------------------------------ gated DeltaNet

@pytest.mark.parametrize("shape", [(1, 64, 16, 128), (2, 3, 16, 128), (1, 5, 4, 64), (3, 1, 7, 32), (1, 2, 3, 256)])
def test_qk_condition_bit_exact(qvex, shape):
    """engine/model.py:275-277 conditioning: bit-exact with the oracle (same fp32 sum order
    and the same two bf16 roundings); row counts that do not fill a 128-row block."""
    q = O.f32_to_bf16(detrand.normal(shape, 61) * 3.0)
    k = O.f32_to_bf16(detrand.normal(shape, 62) * 0.01)
    rq, rk = O.qk_condition(q, k)
    gq, gk = qvex.qk_condition(dev(q), dev(k))
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(gq), rq) and np.array_equal(host_u16(gk), rk)


def test_qk_condition_in_place_and_zero_rows(qvex):
    import ctypes
    from qvex import _lib
    q = O.f32_to_bf16(detrand.normal((300, 128), 63))
    k = O.f32_to_bf16(detrand.normal((300, 128), 64))
    rq, rk = O.qk_condition(q, k)
    qd, kd = dev(q), dev(k)
    P = ctypes.c_void_p
    s = P(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib().qvx_qk_condition(P(qd.data_ptr()), P(kd.data_ptr()), P(qd.data_ptr()),
                                           P(kd.data_ptr()), 300, 128, s), "qk")
    assert _lib.lib().qvx_qk_condition(P(qd.data_ptr()), P(kd.data_ptr()), P(qd.data_ptr()),
                                       P(kd.data_ptr()), 0, 128, s) == 0
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(qd), rq) and np.array_equal(host_u16(kd), rk)

def run_gd(qvex, q, k, v, a, b, A_log, dt, st, keep_mid):
    outs = qvex.gated_delta(dev(q), dev(k), dev(v), dev(a), dev(b), torch.from_numpy(A_log).cuda(),
                            torch.from_numpy(dt).cuda(), torch.from_numpy(st).cuda(), keep_mid=keep_mid)
    torch.cuda.synchronize()
    return [host_u16(outs[0])] + [o.cpu().numpy() for o in outs[1:]]


@pytest.mark.parametrize("name", sorted(p.name for p in __import__("conftest").GOLDEN.glob("gd_b*.npz")))
def test_gated_delta_matches_reference_kernel_fixture(qvex, golden_dir, name):
    z = np.load(golden_dir / name)
    mid = "state_mid" in z.files
    out = run_gd(qvex, z["q"], z["k"], z["v"], z["a"], z["b"], z["A_log"], z["dt_bias"], z["state"], mid)
    assert rel_l2(out[0], z["y"]) <= MATMUL_TOL
    assert rel_l2(out[1], z["state_out"]) <= STATE_TOL
    if mid:
        assert rel_l2(out[2], z["state_mid"]) <= STATE_TOL


@pytest.mark.parametrize("kind", ["zeros", "normal"])
def test_gated_delta_qwen35_fixture(qvex, golden_dir, kind):
    z = np.load(golden_dir / f"gd_qwen35_t4_{kind}.npz")
    q, k, v, a, b, st = gd_inputs(1, 4, 16, 32, 128, 128, int(z["seed"]), kind)
    zeros = np.zeros(32, np.float32)
    y, so, sm = run_gd(qvex, q, k, v, a, b, zeros, zeros, st, True)
    assert rel_l2(y, z["y"]) <= MATMUL_TOL
    assert rel_l2(so.reshape(-1)[::4099], z["state_out_sample"]) <= STATE_TOL


@pytest.mark.parametrize("B,T,kind", [(1, 1, "normal"), (8, 1, "normal"), (1, 2048, "zeros"), (8, 64, "normal"),
                                      (2, 2, "zeros")])
def test_gated_delta_config3_vs_oracle(qvex, B, T, kind):
    q, k, v, a, b, st = gd_inputs(B, T, 16, 32, 128, 128, 900 + B + T, kind)
    zeros = np.zeros(32, np.float32)
    ry, rs = O.gated_delta(q, k, v, a, b, zeros, zeros, st)
    y, so = run_gd(qvex, q, k, v, a, b, zeros, zeros, st, False)
    assert rel_l2(y, ry) <= MATMUL_TOL
    assert rel_l2(so, rs) <= STATE_TOL


def test_gated_delta_snapshot_rollback(qvex):
    """Config 3: 4 steps with the snapshot; state_mid must equal the state after 3 steps
    from the same kernel (bitwise) and re-running step 4 from it must reproduce state_out."""
    q, k, v, a, b, st = gd_inputs(1, 4, 16, 32, 128, 128, 1234, "normal")
    zeros = np.zeros(32, np.float32)
    y4, s4, mid = run_gd(qvex, q, k, v, a, b, zeros, zeros, st, True)
    y3, s3 = run_gd(qvex, q[:, :3], k[:, :3], v[:, :3], a[:, :3], b[:, :3], zeros, zeros, st, False)
    assert np.array_equal(mid, s3)
    assert np.array_equal(y4[:, :3], y3)
    y_last, s_again = run_gd(qvex, q[:, 3:], k[:, 3:], v[:, 3:], a[:, 3:], b[:, 3:], zeros, zeros, mid, False)
    assert np.array_equal(s_again, s4)
    assert np.array_equal(y_last[:, 0], y4[:, 3])


def test_gated_delta_gates_and_gqa_dk64(qvex):
    q, k, v, a, b, st = gd_inputs(2, 9, 2, 8, 64, 32, 55, "normal")
    A_log = (detrand.normal((8,), 56) * 0.5).astype(np.float32)
    dt = (detrand.normal((8,), 57) * 3.0).astype(np.float32)  # softplus linear branch (x > 20) is reached
    a = O.f32_to_bf16(O.bf16_to_f32(a) * 12.0)
    ry, rs, rm = O.gated_delta(q, k, v, a, b, A_log, dt, st, keep_mid=True)
    y, so, sm = run_gd(qvex, q, k, v, a, b, A_log, dt, st, True)
    assert rel_l2(y, ry) <= MATMUL_TOL
    assert rel_l2(so, rs) <= STATE_TOL and rel_l2(sm, rm) <= STATE_TOL


def test_gated_delta_in_place_state(qvex):
    q, k, v, a, b, st = gd_inputs(1, 3, 16, 32, 128, 128, 77, "normal")
    zeros = torch.zeros(32, device="cuda")
    state = torch.from_numpy(st).cuda()
    y1, s1 = qvex.gated_delta(dev(q), dev(k), dev(v), dev(a), dev(b), zeros, zeros, state)
    y2, s2 = qvex.gated_delta(dev(q), dev(k), dev(v), dev(a), dev(b), zeros, zeros, state, out_state=state)
    assert s2.data_ptr() == state.data_ptr()
    assert torch.equal(s1, s2) and torch.equal(y1, y2)


@pytest.mark.parametrize("B,T,Hk,Hv,D", [(1, 40, 16, 32, 128), (3, 17, 4, 8, 64), (2, 100, 2, 4, 32)])
def test_gated_delta_chunked_equals_per_step(qvex, B, T, Hk, Hv, D):
    """T >= 16 runs the kernel that stages q, k, v, a, b through shared memory a chunk ahead;
    a and b that are not 4-byte aligned take the per-step kernel instead.  Both give the same
    bits (outputs, state, pre-last-step snapshot), with gates from A_log / dt_bias != 0."""
    q, k, v, a, b, st = gd_inputs(B, T, Hk, Hv, D, D, 5 + T, "normal")
    g = torch.Generator(device="cuda").manual_seed(T)
    A_log = torch.randn(Hv, device="cuda", generator=g) * 0.5
    dt = torch.randn(Hv, device="cuda", generator=g) * 0.5
    state = torch.from_numpy(st).cuda()
    ad, bd = dev(a), dev(b)
    # the same values one bf16 element into a larger buffer: 2-byte aligned
    a2 = torch.empty(ad.numel() + 1, dtype=torch.bfloat16, device="cuda")[1:].view(ad.shape)
    b2 = torch.empty(bd.numel() + 1, dtype=torch.bfloat16, device="cuda")[1:].view(bd.shape)
    a2.copy_(ad)
    b2.copy_(bd)
    assert a2.data_ptr() % 4 == 2
    r1 = qvex.gated_delta(dev(q), dev(k), dev(v), ad, bd, A_log, dt, state, keep_mid=True)
    r2 = qvex.gated_delta(dev(q), dev(k), dev(v), a2, b2, A_log, dt, state, keep_mid=True)
    for x1, x2 in zip(r1, r2):
        assert torch.equal(x1, x2)


# ------------------------------------------------------------------ qmm (tensor cores, M > 8)

def qmm_direct(qvex, x, w, s, b, short_by=0):
    """Call qvx_qmm through the C ABI for any M (including M <= 8), with a workspace
    `short_by` bytes smaller than qvx_qmm_workspace_size asks for."""
    import ctypes
    from qvex import _lib
    M, K = x.shape
    N = w.shape[0]
    xd, wd, sd, bd = dev(x), dev(w), dev(s), dev(b)
    y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    need = _lib.lib().qvx_qmm_workspace_size(M, N, K) - short_by
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    P = ctypes.c_void_p
    rc = _lib.lib().qvx_qmm(P(xd.data_ptr()), P(wd.data_ptr()), P(sd.data_ptr()), P(bd.data_ptr()),
                            P(y.data_ptr()), M, N, K, 64, 4, P(ws.data_ptr()), need,
                            P(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "qvx_qmm")
    torch.cuda.synchronize()
    return host_u16(y)


@pytest.mark.parametrize("M,N,K", [(9, 256, 64), (48, 384, 192), (130, 640, 320), (16, 256, 1024),
                                   (64, 1024, 4096), (100, 300, 512), (40, 300, 512), (63, 257, 2048),
                                   (129, 520, 1024), (256, 257, 2048), (512, 4096, 4096), (37, 12288, 4096),
                                   (200, 4096, 12288)])
def test_qmm_matches_oracle(qvex, M, N, K):
    x, _, w, s, b = qmv_inputs(M, K, N, seed=7 * M + N + K)
    ref = O.qmm_exact(x, w, s, b)
    y = qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b))
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y), ref) <= MATMUL_TOL


@pytest.mark.parametrize("M", [1, 2, 5, 8])
def test_qmm_small_m_direct(qvex, M):
    x, _, w, s, b = qmv_inputs(M, 2048, 384, seed=300 + M)
    ref = O.qmm_exact(x, w, s, b)
    assert rel_l2(qmm_direct(qvex, x, w, s, b), ref) <= MATMUL_TOL


@pytest.mark.parametrize("M,N,K", [(64, 1024, 4096), (16, 12288, 4096), (128, 4096, 12288), (33, 520, 2048)])
def test_qmm_k_split_matches_unsplit(qvex, M, N, K):
    """Small M: the tiles do not fill the SMs, so qvx_qmm splits K across SMs and sums
    fp32 partials in the workspace.  A workspace without room for the partials (one byte
    short) runs the unsplit kernel; both agree with the oracle and with each other."""
    x, _, w, s, b = qmv_inputs(M, K, N, seed=11 * M + N + K)
    ref = O.qmm_exact(x, w, s, b)
    split = qmm_direct(qvex, x, w, s, b)
    whole = qmm_direct(qvex, x, w, s, b, short_by=1)
    assert rel_l2(split, ref) <= MATMUL_TOL
    assert rel_l2(whole, ref) <= MATMUL_TOL
    assert rel_l2(split, whole) <= MATMUL_TOL


def test_qmm_config2_full_size_sampled(qvex):
    """Config 2: W ~ N(0, 0.02) [12288, 4096] quantised, x ~ N(0,1) [2048, 4096]; the
    oracle checks every 16th token row (all 12288 outputs of each)."""
    W = O.f32_to_bf16(detrand.normal((12288, 4096), 2) * 0.02)
    wq, s, b = O.quantize(W, 64, "minmax")
    x = O.f32_to_bf16(detrand.normal((2048, 4096), 3))
    y = qvex.quantized_matmul(dev(x), dev(wq), dev(s), dev(b))
    torch.cuda.synchronize()
    yh = host_u16(y)
    ref = O.qmm_exact(x[::16], wq, s, b)
    assert rel_l2(yh[::16], ref) <= MATMUL_TOL
    assert np.isfinite(O.bf16_to_f32(yh)).all()


def test_qmm_dynamic_range(qvex):
    """Token rows and weight rows whose magnitudes differ by many orders: the per-row
    power-of-two scaling keeps fp16 operands in range without losing precision."""
    M, N, K = 48, 320, 1024
    x = detrand.normal((M, K), 5)
    x[0] *= 3e4      # would overflow fp16 unscaled
    x[1] *= 1e-6     # would underflow
    x[2] = 0.0       # all-zero row
    xb = O.f32_to_bf16(x)
    W = detrand.normal((N, K), 6) * 0.02
    W[0] *= 1e3
    W[1] *= 1e-5
    W[2, :64] = 0.0
    wq, s, b = O.quantize(O.f32_to_bf16(W), 64, "minmax")
    ref = O.qmm_exact(xb, wq, s, b)
    y = host_u16(qvex.quantized_matmul(dev(xb), dev(wq), dev(s), dev(b)))
    r = O.bf16_to_f32(ref).astype(np.float64)
    g = O.bf16_to_f32(y).astype(np.float64)
    assert np.all(g[2] == 0)
    # per token row relative error (row scales differ by 1e10)
    for m in (0, 1, 3):
        assert np.linalg.norm(g[m] - r[m]) / np.linalg.norm(r[m]) <= MATMUL_TOL
    # per weight row
    for n in (0, 1, 5):
        assert np.linalg.norm(g[:, n] - r[:, n]) / np.linalg.norm(r[:, n]) <= 2 * MATMUL_TOL


def test_qmm_and_qmv_agree(qvex):
    x, _, w, s, b = qmv_inputs(8, 4096, 1024, seed=99)
    y_qmv = host_u16(qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b)))
    y_qmm = qmm_direct(qvex, x, w, s, b)
    assert rel_l2(y_qmm, y_qmv) <= MATMUL_TOL


@pytest.mark.parametrize("M,N,K", [(64, 1024, 4096), (16, 300, 192), (200, 4096, 1024), (33, 520, 2048),
                                   (64, 12352, 4096)])
def test_qmm_prepared_equals_qmm(qvex, M, N, K):
    """qvx_qmm_prepared with a prepass made once by qvx_qmm_prepare gives qvx_qmm's bits,
    twice in a row with the same buffer; QLinear takes that path above QMV_MAX_M rows."""
    x, _, w, s, b = qmv_inputs(M, K, N, seed=17 * M + N + K)
    xd, wd, sd, bd = dev(x), dev(w), dev(s), dev(b)
    ref = host_u16(qvex.quantized_matmul(xd, wd, sd, bd))
    prep = qvex.core.qmm_prepare(sd, bd)
    for _ in range(2):
        got = host_u16(qvex.quantized_matmul(xd, wd, sd, bd, prep=prep))
        assert np.array_equal(got, ref)
    lin = qvex.QLinear(wd, sd, bd)
    assert np.array_equal(host_u16(lin(xd)), ref)
    assert lin.prepared() is not None


def test_qmm_workspace_reuse_and_out(qvex):
    x, _, w, s, b = qmv_inputs(64, 1024, 512, seed=4)
    ref = O.qmm_exact(x, w, s, b)
    need = qvex.qmm_workspace_size(64, 512, 1024)
    ws = torch.empty(need + 4096, dtype=torch.uint8, device="cuda")
    out = torch.empty(64, 512, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b), out=out, workspace=ws)
    assert rel_l2(host_u16(out), ref) <= MATMUL_TOL


# ------------------------------------------------------------------ every shape of the benchmark's decode step

CONFIG1_SHAPES = [(12352, 4096), (4096, 4096), (8192, 4096), (1024, 4096), (10240, 4096), (24576, 4096),
                  (4096, 12288)]  # in_proj, out/o_proj, q_proj, k/v_proj, fused q|k|v, gate_up, down


@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("N,K", CONFIG1_SHAPES)
def test_qmv_config1_shapes(qvex, M, N, K):
    """Every distinct projection shape of the Qwen3.5-9B decode step at the verify widths
    M = 1, 2, 4, 8 (the streaming kernel's one- and two-token plans, all row tilings)."""
    x, _, w, s, b = qmv_inputs(M, K, N, seed=7 * M + N + K)
    y = qvex.quantized_matmul(dev(x), dev(w), dev(s), dev(b))
    ref = O.qmm_exact(x, w, s, b)
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y), ref) <= MATMUL_TOL


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_qmv_lm_head_sampled(qvex, M):
    """lm_head [248320, 4096] (572 MB, one launch) at M = 1, 2, 4, 8; the oracle checks every
    97th output row (2560 rows, all M tokens)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(M)
    N, K = 248320, 4096
    w = torch.randint(-2 ** 31, 2 ** 31, (N, K // 8), dtype=torch.int64, device="cuda", generator=g).to(torch.int32)
    s = (torch.randn((N, K // 64), device="cuda", generator=g).abs() * 0.002).to(torch.bfloat16)
    b = (-8.0 * s.float()).to(torch.bfloat16)
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    y = qvex.quantized_matmul(x, w, s, b)
    rows = slice(None, None, 97)
    ref = O.qmm_exact(host_u16(x), w[rows].cpu().numpy().view(np.uint32), host_u16(s[rows]), host_u16(b[rows]))
    torch.cuda.synchronize()
    assert rel_l2(host_u16(y[:, rows].contiguous()), ref) <= MATMUL_TOL


def test_gated_delta_config3_b8_t2048_with_rollback(qvex):
    """Config 3 at its benchmarked size: B = 8, T = 2048, N(0,1)*0.1 state, A_log = dt_bias = 0;
    y and the final state against the oracle, and the snapshot before the last step
    reproduces the final state when the last step is rerun from it (bitwise)."""
    g = torch.Generator().manual_seed(77)
    B, T, Hk, Hv, D = 8, 2048, 16, 32, 128

    def bf16(t):
        return O.f32_to_bf16(t.numpy().astype(np.float32))
    q = bf16(torch.nn.functional.normalize(torch.randn((B, T, Hk, D), generator=g), dim=-1))
    k = bf16(torch.nn.functional.normalize(torch.randn((B, T, Hk, D), generator=g), dim=-1))
    v = bf16(torch.randn((B, T, Hv, D), generator=g))
    a = bf16(torch.randn((B, T, Hv), generator=g))
    b = bf16(torch.randn((B, T, Hv), generator=g))
    st = (torch.randn((B, Hv, D, D), generator=g) * 0.1).numpy()
    zeros = np.zeros(Hv, np.float32)
    y, so, sm = run_gd(qvex, q, k, v, a, b, zeros, zeros, st, True)
    ry, rs = O.gated_delta(q, k, v, a, b, zeros, zeros, st)
    assert rel_l2(y, ry) <= MATMUL_TOL
    assert rel_l2(so, rs) <= STATE_TOL
    # rerun the last step from the snapshot
    last = [np.ascontiguousarray(t[:, -1:]) for t in (q, k, v, a, b)]
    y2, so2 = run_gd(qvex, *last, zeros, zeros, sm, False)
    assert np.array_equal(so2, so) and np.array_equal(y2, y[:, -1:])
