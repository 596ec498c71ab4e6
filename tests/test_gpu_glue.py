"""Decoder-layer glue kernels (qvx_rms_norm, qvx_gated_rms_norm, qvx_swiglu,
qvx_deltanet_conv, qvx_attention) against the CPU oracle (oracle/model_oracle.c) on seeded
inputs, through the C ABI.

Bars: results without a transcendental function (rms_norm with the residual add, the conv
state windows, the a/b copies, the value cache) bit for bit; results through exp, sin or cos
(CUDA's and the C library's differ by an ulp) within rel-L2 1e-3 of bf16 outputs, with at
least 98 % of the elements bit-equal."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.bfloat16)
    return t.cuda()


def host(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def bf(rng, shape, scale=1.0):
    return O.f32_to_bf16(rng.standard_normal(shape).astype(np.float32) * scale)


def close(got, ref, rel=1e-3, frac=0.98):
    g, r = O.bf16_to_f32(got).astype(np.float64), O.bf16_to_f32(ref).astype(np.float64)
    err = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    same = np.mean(got == ref)
    assert err <= rel and same >= frac, f"rel-L2 {err:.2e}, bit-equal {same:.4f}"


@pytest.mark.parametrize("M,D", [(1, 4096), (3, 4096), (64, 4096), (5, 128), (2, 12288)])
@pytest.mark.parametrize("with_resid", [False, True])
def test_rms_norm_bit_exact(M, D, with_resid):
    import qvex.glue as G
    rng = np.random.default_rng(M * 7 + D)
    x, r = bf(rng, (M, D), 3.0), bf(rng, (M, D))
    w = bf(rng, (D,), 0.5)
    if with_resid:
        out, h = G.rms_norm(dev(x), dev(w), 1e-6, resid=dev(r))
        ro, rh = O.rms_norm(x, w, 1e-6, resid=r)
        assert np.array_equal(host(h), rh)
    else:
        out = G.rms_norm(dev(x), dev(w), 1e-6)
        ro = O.rms_norm(x, w, 1e-6)
    assert np.array_equal(host(out), ro)


def test_rms_norm_in_place_and_unweighted():
    import qvex.glue as G
    rng = np.random.default_rng(3)
    x, r = bf(rng, (4, 4096)), bf(rng, (4, 4096))
    xt, rt = dev(x), dev(r)
    out, h = G.rms_norm(xt, None, 1e-5, resid=rt, h_out=rt)  # residual stream updated in place
    ro, rh = O.rms_norm(x, None, 1e-5, resid=r)
    assert np.array_equal(host(rt), rh) and np.array_equal(host(out), ro)


@pytest.mark.parametrize("T", [1, 7])
def test_gated_rms_norm(T):
    import qvex.glue as G
    rng = np.random.default_rng(T)
    H, D, stride = 32, 128, 12352
    y = bf(rng, (T, H, D))
    proj = bf(rng, (T, stride))
    w = bf(rng, (D,), 0.3)
    z = dev(proj)[:, 8192:8192 + H * D]  # the z columns of an in_proj output row
    got = G.gated_rms_norm(dev(y), z, dev(w), 1e-6)
    ref = O.gated_rms_norm(y, np.ascontiguousarray(proj[:, 8192:8192 + H * D]), w, 1e-6)
    close(host(got), ref)


@pytest.mark.parametrize("M,I", [(1, 12288), (3, 12288), (64, 1024)])
def test_swiglu(M, I):
    import qvex.glue as G
    rng = np.random.default_rng(M + I)
    gu = bf(rng, (M, 2 * I), 2.0)
    close(host(G.swiglu(dev(gu))), O.swiglu(gu))


CONV_SHAPES = [(16, 32, 128), (2, 4, 128), (1, 2, 64)]  # Hk, Hv, D


@pytest.mark.parametrize("B,T", [(1, 1), (3, 1), (1, 2), (2, 5), (1, 130)])
@pytest.mark.parametrize("Hk,Hv,D", CONV_SHAPES)
def test_deltanet_conv(B, T, Hk, Hv, D):
    import qvex.glue as G
    rng = np.random.default_rng(B * 100 + T + D)
    C = 2 * Hk * D + Hv * D
    S = C + Hv * D + 2 * Hv + 6  # an in_proj row (plus slack, as a strided view would have)
    proj = bf(rng, (B, T, S))
    conv_w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    st = bf(rng, (B, 3, C))
    keep = T >= 2
    got = G.deltanet_conv(dev(proj), dev(conv_w), dev(st), Hk, Hv, D, D, keep_mid=keep)
    ref = O.deltanet_conv(proj, conv_w, st, Hk, Hv, D, D, keep_mid=keep)
    for name, g, r in zip("qkv", got[:3], ref[:3]):
        close(host(g), r)
    assert np.array_equal(host(got[3]), ref[3]) and np.array_equal(host(got[4]), ref[4]), "a/b copies differ"
    assert np.array_equal(host(got[5]), ref[5]), "state_out differs"
    if keep:
        assert np.array_equal(host(got[6]), ref[6]), "state_mid differs"


def test_deltanet_conv_in_place_state():
    import qvex.glue as G
    rng = np.random.default_rng(9)
    Hk, Hv, D = 16, 32, 128
    C = 2 * Hk * D + Hv * D
    proj = bf(rng, (2, 1, C + Hv * D + 2 * Hv))
    conv_w = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    st = bf(rng, (2, 3, C))
    stt = dev(st)
    got = G.deltanet_conv(dev(proj), dev(conv_w), stt, Hk, Hv, D, D, state_out=stt)
    ref = O.deltanet_conv(proj, conv_w, st, Hk, Hv, D, D)
    assert np.array_equal(host(stt), ref[5])
    close(host(got[0]), ref[0])


ATT = dict(H=32, Hkv=8, D=128, rd=32, base=1e7)


def _attn_case(rng, B, L, pos, cap, H=32, Hkv=8, D=128):
    qkv = bf(rng, (B, L, (2 * H + 2 * Hkv) * D))
    qn, kn = bf(rng, (D,), 0.2), bf(rng, (D,), 0.2)
    kc = bf(rng, (B, Hkv, cap, D))  # positions [0, pos) hold earlier tokens
    vc = bf(rng, (B, Hkv, cap, D))
    return qkv, qn, kn, kc, vc


@pytest.mark.parametrize("B,L,pos", [(1, 1, 0), (1, 1, 37), (1, 1, 1000), (3, 1, 300), (1, 2, 77), (2, 2, 4095)])
def test_attention_decode_split_keys(B, L, pos):
    import qvex.glue as G
    rng = np.random.default_rng(B * 1000 + L + pos)
    cap = 4097 + 3
    qkv, qn, kn, kc, vc = _attn_case(rng, B, L, pos, cap)
    kct, vct = dev(kc), dev(vc)
    inv = G.rope_inv_freq(ATT["rd"], ATT["base"], "cuda")
    ws = G.attention_workspace(B, 8, 4, L, 128, 16, "cuda")
    assert ws is not None
    outs = []
    for _ in range(2):  # twice: the workspace counters must come back to zero
        outs.append(host(G.attention(dev(qkv), dev(qn), dev(kn), 1e-6, inv, kct, vct, pos, 32, 8, 128,
                                     workspace=ws, nsplit=16)))
    ro = O.attention(qkv, qn, kn, kc, vc, pos, 32, 8, 128, ATT["rd"], ATT["base"])
    assert np.array_equal(outs[0], outs[1])
    close(outs[0], ro)
    assert np.array_equal(host(vct), vc), "value cache differs"
    close(host(kct)[:, :, pos:pos + L], kc[:, :, pos:pos + L])
    assert np.array_equal(host(kct)[:, :, :pos], kc[:, :, :pos])


def test_attention_position_from_device_memory():
    import qvex.glue as G
    rng = np.random.default_rng(5)
    qkv, qn, kn, kc, vc = _attn_case(rng, 1, 1, 50, 256)
    inv = G.rope_inv_freq(32, 1e7, "cuda")
    ws = G.attention_workspace(1, 8, 4, 1, 128, 8, "cuda")
    pos = torch.tensor([50], dtype=torch.int32, device="cuda")
    kct, vct = dev(kc), dev(vc)
    got = G.attention(dev(qkv), dev(qn), dev(kn), 1e-6, inv, kct, vct, pos, 32, 8, 128, workspace=ws, nsplit=8)
    kc2, vc2 = kc.copy(), vc.copy()
    ref = host(G.attention(dev(qkv), dev(qn), dev(kn), 1e-6, inv, dev(kc2), dev(vc2), 50, 32, 8, 128, workspace=ws,
                           nsplit=8))
    assert np.array_equal(host(got), ref)


@pytest.mark.parametrize("B,L,pos", [(1, 70, 0), (2, 33, 10), (1, 9, 500)])
def test_attention_prefill(B, L, pos):
    import qvex.glue as G
    rng = np.random.default_rng(B + L + pos)
    cap = pos + L + 5
    qkv, qn, kn, kc, vc = _attn_case(rng, B, L, pos, cap)
    kct, vct = dev(kc), dev(vc)
    inv = G.rope_inv_freq(ATT["rd"], ATT["base"], "cuda")
    got = G.attention(dev(qkv), dev(qn), dev(kn), 1e-6, inv, kct, vct, pos, 32, 8, 128)
    ro = O.attention(qkv, qn, kn, kc, vc, pos, 32, 8, 128, ATT["rd"], ATT["base"])
    close(host(got), ro)
    assert np.array_equal(host(vct), vc)


def test_attention_small_heads():
    """D = 64, two query heads per KV head, a partial rotary span: the general shapes."""
    import qvex.glue as G
    rng = np.random.default_rng(11)
    B, L, pos, H, Hkv, D, rd = 2, 1, 20, 4, 2, 64, 16
    qkv, qn, kn, kc, vc = _attn_case(rng, B, L, pos, 64, H, Hkv, D)
    kct, vct = dev(kc), dev(vc)
    inv = G.rope_inv_freq(rd, 1e4, "cuda")
    ws = G.attention_workspace(B, Hkv, H // Hkv, L, D, 4, "cuda")
    got = G.attention(dev(qkv), dev(qn), dev(kn), 1e-6, inv, kct, vct, pos, H, Hkv, D, workspace=ws, nsplit=4)
    ro = O.attention(qkv, qn, kn, kc, vc, pos, H, Hkv, D, rd, 1e4)
    close(host(got), ro)
