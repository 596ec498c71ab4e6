"""qvx_deltanet_decode (conv, recurrence and gated norm in one kernel) against the three
kernels it fuses (qvx_deltanet_conv, qvx_gated_delta, qvx_gated_rms_norm) on the same seeded
inputs: every output bit for bit -- the out_proj input, the new conv window, the new
recurrent state and both pre-last-token snapshots -- in place and out of place."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(B, T, Hk, Hv, Dk, Dv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    C = 2 * Hk * Dk + Hv * Dv
    S = C + Hv * Dv + 2 * Hv + 24  # a row stride past the packed width
    proj = torch.randn((B, T, S), device="cuda", generator=g).to(torch.bfloat16)
    conv_w = torch.randn((C, 4), device="cuda", generator=g) * 0.5
    conv = torch.randn((B, 3, C), device="cuda", generator=g).to(torch.bfloat16)
    A_log = torch.randn(Hv, device="cuda", generator=g) * 0.5
    dt_bias = torch.randn(Hv, device="cuda", generator=g) * 0.5
    state = torch.randn((B, Hv, Dv, Dk), device="cuda", generator=g) * 0.1
    norm_w = (1.0 + 0.1 * torch.randn(Dv, device="cuda", generator=g)).to(torch.bfloat16)
    return proj, conv_w, conv, A_log, dt_bias, state, norm_w


def _three_kernels(proj, conv_w, conv, A_log, dt_bias, state, norm_w, Hk, Hv, Dk, Dv, keep):
    from qvex import glue
    from qvex.kernels import gated_delta
    B, T, _ = proj.shape
    C = 2 * Hk * Dk + Hv * Dv
    r = glue.deltanet_conv(proj, conv_w, conv, Hk, Hv, Dk, Dv, keep_mid=keep)
    q, k, v, a, b, conv_out = r[:6]
    gd = gated_delta(q, k, v, a, b, A_log, dt_bias, state, keep_mid=keep)
    z = proj.reshape(B * T, -1)[:, C:C + Hv * Dv]
    out = glue.gated_rms_norm(gd[0], z, norm_w, 1e-6).view(B, T, Hv * Dv)
    return out, conv_out, gd[1], (r[6] if keep else None), (gd[2] if keep else None)


@pytest.mark.parametrize("B,T,Hk,Hv,Dk,Dv", [(1, 1, 16, 32, 128, 128), (3, 1, 16, 32, 128, 128),
                                             (1, 2, 16, 32, 128, 128), (2, 4, 2, 4, 128, 128),
                                             (2, 3, 2, 8, 64, 64)])
@pytest.mark.parametrize("keep", [False, True])
def test_fused_equals_three_kernels(B, T, Hk, Hv, Dk, Dv, keep):
    from qvex import glue
    if not glue.deltanet_decode_supported(T, Hk, Hv, Dk, Dv):
        pytest.skip("shape outside the fused kernel")
    proj, conv_w, conv, A_log, dt_bias, state, norm_w = _case(B, T, Hk, Hv, Dk, Dv, 7 + B + T)
    ref = _three_kernels(proj, conv_w, conv, A_log, dt_bias, state, norm_w, Hk, Hv, Dk, Dv, keep)
    got = glue.deltanet_decode(proj, conv_w, conv, A_log, dt_bias, state, norm_w, 1e-6, Hk, Hv, Dk, Dv, keep_mid=keep)
    names = ["out", "conv_out", "state_out", "conv_mid", "state_mid"]
    for name, x, y in zip(names, got, ref):
        if y is None:
            continue
        assert torch.equal(x.view(torch.int16) if x.dtype == torch.bfloat16 else x.view(torch.int32),
                           y.view(torch.int16) if y.dtype == torch.bfloat16 else y.view(torch.int32)), name


def test_fused_in_place_updates():
    """conv_out / state_out given as the input buffers: the same bits as out of place."""
    from qvex import glue
    B, T, Hk, Hv, Dk, Dv = 2, 2, 16, 32, 128, 128
    proj, conv_w, conv, A_log, dt_bias, state, norm_w = _case(B, T, Hk, Hv, Dk, Dv, 3)
    ref = glue.deltanet_decode(proj, conv_w, conv, A_log, dt_bias, state, norm_w, 1e-6, Hk, Hv, Dk, Dv, keep_mid=True)
    c2, s2 = conv.clone(), state.clone()
    got = glue.deltanet_decode(proj, conv_w, c2, A_log, dt_bias, s2, norm_w, 1e-6, Hk, Hv, Dk, Dv, conv_out=c2,
                               state_out=s2, keep_mid=True)
    assert got[1].data_ptr() == c2.data_ptr() and got[2].data_ptr() == s2.data_ptr()
    for x, y in zip(got, ref):
        assert torch.equal(x, y)


def test_unsupported_shape_is_refused():
    from qvex import glue
    B, T, Hk, Hv, Dk, Dv = 1, 5, 16, 32, 128, 128  # T > 4
    proj, conv_w, conv, A_log, dt_bias, state, norm_w = _case(B, T, Hk, Hv, Dk, Dv, 1)
    assert not glue.deltanet_decode_supported(T, Hk, Hv, Dk, Dv)
    with pytest.raises(NotImplementedError):
        glue.deltanet_decode(proj, conv_w, conv, A_log, dt_bias, state, norm_w, 1e-6, Hk, Hv, Dk, Dv)


def test_model_fused_equals_unfused():
    """A small model's decode steps with the fused DeltaNet kernel and with the three kernels
    give the same logits bit for bit (plain steps and a 2-token keep_prev verify)."""
    from test_model_oracle import small_cfg
    from qvex.qwen35 import GatedDeltaNet, Qwen35, random_params
    cfg = small_cfg()
    model = Qwen35.from_params(cfg, random_params(cfg, 5, "cuda"))
    prompt = torch.randint(0, cfg.vocab_size, (2, 9), device="cuda", dtype=torch.int32,
                           generator=torch.Generator(device="cuda").manual_seed(2))
    steps = [torch.randint(0, cfg.vocab_size, (2, L), device="cuda", dtype=torch.int32,
                           generator=torch.Generator(device="cuda").manual_seed(10 + i)) for i, L in enumerate((1, 1, 2, 1))]
    outs = []
    for fused in (True, False):
        GatedDeltaNet.fused_decode = fused
        try:
            cache = model.make_cache()
            seq = [model(prompt, cache, last_only=True)]
            for i, ids in enumerate(steps):
                seq.append(model(ids, cache, last_only=False, keep_prev=ids.shape[1] == 2))
            outs.append(seq)
        finally:
            GatedDeltaNet.fused_decode = True
    for a, b in zip(*outs):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
