"""Fused decode projections (qvx_qmv_fused) on one GPU, through the C ABI.

Each prologue must give exactly the bits of the standalone glue kernel followed by the
plain decode projection (the prologues reuse the glue kernels' arithmetic and reduction
order), and the residual epilogue exactly the bits of the residual add:
  rms_norm        == qvx_rms_norm -> qvx_qmv            (decoder-layer input norms, final norm)
  swiglu          == qvx_swiglu -> qvx_qmv              (MLP down projection)
  gated_rms_norm  == qvx_gated_rms_norm -> qvx_qmv      (DeltaNet out_proj)
  resid           == qvx_qmv -> bf16(resid + y)         (in place on the residual stream)
and the whole fused decode step of the model against the unfused one (logits bit-equal)."""
import numpy as np
import pytest
import torch

from make_golden import qmv_inputs

pytestmark = pytest.mark.gpu


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.bfloat16)
    elif a.dtype == np.uint32:
        t = t.view(torch.int32)
    return t.cuda()


def same(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def weights(N, K, seed):
    _, _, w, s, b = qmv_inputs(1, K, N, seed)
    return dev(w), dev(s), dev(b)


@pytest.mark.parametrize("M", [1, 2, 3, 8])
@pytest.mark.parametrize("N,K", [(12352, 4096), (1024, 4096), (512, 1536), (640, 512)])
def test_rms_norm_prologue(M, N, K):
    import qvex
    from qvex import glue
    w, s, b = weights(N, K, M + N)
    g = torch.Generator(device="cuda").manual_seed(M)
    x = (torch.randn((M, K), device="cuda", generator=g) * 3).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    got = qvex.core.qmv_fused(x, w, s, b, prologue="rms_norm", norm_w=nw, eps=1e-6)
    ref = qvex.quantized_matmul(glue.rms_norm(x, nw, 1e-6), w, s, b)
    assert same(got, ref)


@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("N,K", [(4096, 12288), (4096, 1536), (512, 1024)])
def test_swiglu_prologue(M, N, K):
    import qvex
    from qvex import glue
    w, s, b = weights(N, K, 3 * M + N)
    g = torch.Generator(device="cuda").manual_seed(M)
    gu = (torch.randn((M, 2 * K), device="cuda", generator=g) * 2).to(torch.bfloat16)
    got = qvex.core.qmv_fused(gu, w, s, b, prologue="swiglu")
    ref = qvex.quantized_matmul(glue.swiglu(gu), w, s, b)
    assert same(got, ref)


@pytest.mark.parametrize("M", [1, 2, 4])
@pytest.mark.parametrize("N,K,stride,zoff", [(4096, 4096, 12352, 8192), (512, 512, 1544, 1024)])
def test_gated_rms_norm_prologue_and_residual(M, N, K, stride, zoff):
    import qvex
    from qvex import glue
    w, s, b = weights(N, K, 5 * M + N)
    g = torch.Generator(device="cuda").manual_seed(M)
    y = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    proj = torch.randn((M, stride), device="cuda", generator=g).to(torch.bfloat16)  # in_proj rows
    z = proj[:, zoff:zoff + K]
    nw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    resid = torch.randn((M, N), device="cuda", generator=g).to(torch.bfloat16)
    ref_m = qvex.quantized_matmul(glue.gated_rms_norm(y, z, nw, 1e-6), w, s, b)
    ref = glue.add(resid, ref_m)
    got = resid.clone()
    qvex.core.qmv_fused(y, w, s, b, prologue="gated_rms_norm", norm_w=nw, z=z, head_dim=128, eps=1e-6, resid=got,
                        out=got)  # in place on the residual stream
    assert same(got, ref)


def test_plain_with_residual_out_of_place():
    import qvex
    from qvex import glue
    w, s, b = weights(4096, 4096, 9)
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn((2, 4096), device="cuda", generator=g).to(torch.bfloat16)
    resid = torch.randn((2, 4096), device="cuda", generator=g).to(torch.bfloat16)
    got = qvex.core.qmv_fused(x, w, s, b, resid=resid)
    assert same(got, glue.add(resid, qvex.quantized_matmul(x, w, s, b)))


def test_fused_decode_step_equals_unfused():
    """Qwen35.decode_step with the fused projections against the unfused layer glue: the
    same logits, bit for bit, over several steps (small random model)."""
    from qvex.qwen35 import Qwen35, random_params
    from test_model_oracle import small_cfg
    cfg = small_cfg()
    model = Qwen35.from_params(cfg, random_params(cfg, 3, "cuda"))
    B = 3
    ids = torch.randint(0, cfg.vocab_size, (B, 10), device="cuda", dtype=torch.int32)
    caches = [model.make_cache(capacity=32) for _ in range(2)]
    for c in caches:
        model(ids, c, last_only=True)
        model.prepare_decode(c, B, "cuda")
    tok = ids[:, -1:].contiguous()
    pos = torch.tensor([10], dtype=torch.int32, device="cuda")
    for step in range(3):
        a = model.decode_step(tok, caches[0], pos, fused=True)
        b = model.decode_step(tok, caches[1], pos, fused=False)
        assert same(a, b), f"step {step}"
        pos += 1
        tok = a.float().argmax(-1).to(torch.int32).view(B, 1)


@pytest.mark.parametrize("M", [1, 2, 3, 8])
@pytest.mark.parametrize("N,K", [(24576, 4096), (2048, 512), (4096, 12288), (1024, 1536)])
@pytest.mark.parametrize("prologue", ["plain", "rms_norm"])
def test_swiglu_pairs_epilogue(M, N, K, prologue):
    """The gate|up projection with its rows interleaved in (gate, up) pairs and SwiGLU in the
    epilogue == the plain projection over the same rows followed by qvx_swiglu_pairs, and ==
    the [gate | up] projection followed by qvx_swiglu (row order does not change a row)."""
    import qvex
    from qvex import glue
    w, s, b = weights(N, K, 5 * M + N + K)
    g = torch.Generator(device="cuda").manual_seed(M + 7)
    x = (torch.randn((M, K), device="cuda", generator=g) * 2).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    kw = dict(norm_w=nw, eps=1e-6) if prologue == "rms_norm" else {}
    got = qvex.core.qmv_fused(x, w, s, b, prologue=prologue, epilogue="swiglu_pairs", **kw)
    xin = glue.rms_norm(x, nw, 1e-6) if prologue == "rms_norm" else x
    y = qvex.quantized_matmul(xin, w, s, b)
    assert got.shape == (M, N // 2)
    assert same(got, glue.swiglu_pairs(y))
    # the same rows de-interleaved into [gate | up] through qvx_swiglu
    perm = torch.cat([torch.arange(0, N, 2), torch.arange(1, N, 2)]).cuda()
    assert same(got, glue.swiglu(y[:, perm].contiguous()))


def test_swiglu_pairs_epilogue_refusals():
    import qvex
    w, s, b = weights(2048, 512, 1)
    x = torch.randn((1, 512), device="cuda").to(torch.bfloat16)
    r = torch.zeros((1, 2048), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        qvex.core.qmv_fused(x, w, s, b, epilogue="swiglu_pairs", resid=r)
    w3, s3, b3 = weights(2047, 512, 2)
    with pytest.raises(ValueError):
        qvex.core.qmv_fused(x, w3, s3, b3, epilogue="swiglu_pairs")


def test_mlp_interleaved_equals_reference_layout():
    """The model's MLP (interleaved gate|up, SwiGLU in the epilogue at decode, qvx_swiglu_pairs
    at prefill) gives the bits of [gate | up] -> qvx_swiglu -> down."""
    import qvex
    from qvex import glue
    from qvex.model import QLinear
    from qvex.qwen35 import MLP
    H, I = 512, 1024
    gw, gs, gb = weights(I, H, 11)
    uw, us, ub = weights(I, H, 12)
    dw, ds, db = weights(H, I, 13)
    mlp = MLP({"gate_proj": (gw, gs, gb, 64, 4), "up_proj": (uw, us, ub, 64, 4), "down_proj": (dw, ds, db, 64, 4)})
    ref_gu = QLinear.fuse([QLinear(gw, gs, gb, 64, 4), QLinear(uw, us, ub, 64, 4)])
    for M in (1, 4, 40):
        x = torch.randn((M, H), device="cuda", generator=torch.Generator(device="cuda").manual_seed(M)).to(torch.bfloat16)
        ref = qvex.quantized_matmul(glue.swiglu(ref_gu(x)), dw, ds, db)
        assert same(mlp(x), ref), M
