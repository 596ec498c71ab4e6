"""The GPU model (qvex.qwen35.Qwen35 on libqvex) against the CPU model oracle
(oracle/qwen35_oracle.py) on a small random-initialised Qwen3.5-shaped model: 3 gated
DeltaNet layers + 1 gated attention layer, hidden 512, vocab 2048, the 9B model's head
sizes (128) and conv kernel (4).

A sequence runs through every path the reference's engine takes: a 20-token prefill (the
tensor-core projections, the prefill attention kernel, the chunked conv), three decode
steps (the decode projections and the split-key attention), a two-token verify with
keep_prev (engine/speculative.py:72), a rollback of the second token (:98-99) and one more
step; plus batch-2 decode.  Logits are compared after every step: rel-L2 <= 1e-2 of the
bf16 logits (the per-op bar is 1e-3; four layers compound it) and the same argmax on at
least 95 % of the positions."""
import numpy as np
import pytest
import torch

import qwen35_oracle as QO

from test_model_oracle import numpy_params, small_cfg

pytestmark = pytest.mark.gpu

REL = 1e-2


def host(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def rel(got, ref):
    import oracle as O
    g, r = O.bf16_to_f32(got).astype(np.float64), O.bf16_to_f32(ref).astype(np.float64)
    return np.linalg.norm(g - r) / np.linalg.norm(r)


def agree(got, ref):
    import oracle as O
    g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
    return float(np.mean(g.argmax(-1) == r.argmax(-1)))


@pytest.fixture(scope="module")
def models():
    from qvex.qwen35 import Qwen35, random_params
    cfg = small_cfg()
    P = random_params(cfg, 11, "cuda")
    return cfg, Qwen35.from_params(cfg, P), numpy_params(P)


def test_model_prefill_decode_verify_rollback(models):
    cfg, model, P = models
    rng = np.random.default_rng(0)
    ids = rng.integers(0, cfg.vocab_size, (1, 20)).astype(np.int32)
    cache = model.make_cache()
    oc = QO.Cache(cfg, 1, 64)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()
    errs = []

    def step(chunk, keep_prev=False, last_only=False):
        got = host(model(dev(chunk), cache, last_only=last_only, keep_prev=keep_prev))
        ref, _ = QO.forward(cfg, P, chunk, oc, keep_prev=keep_prev)
        if last_only:
            ref = ref[:, -1:]
        e = rel(got, ref)
        errs.append(e)
        assert e <= REL and agree(got, ref) >= 0.95, (len(errs), e, agree(got, ref))

    step(ids)                                        # prefill: every position
    for t in range(3):                               # decode
        step(rng.integers(0, cfg.vocab_size, (1, 1)))
    step(rng.integers(0, cfg.vocab_size, (1, 2)), keep_prev=True)  # verify [last, draft]
    for c in cache:                                  # reject the draft
        c.rollback(1)
    oc.rollback()
    step(rng.integers(0, cfg.vocab_size, (1, 1)), last_only=True)
    print("logit rel-L2 per step:", ["%.1e" % e for e in errs])


def test_model_batched_decode(models):
    cfg, model, P = models
    rng = np.random.default_rng(1)
    B = 2
    cache = model.make_cache()
    oc = QO.Cache(cfg, B, 64)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()
    for L in (9, 1, 1):
        ids = rng.integers(0, cfg.vocab_size, (B, L))
        got = host(model(dev(ids), cache, last_only=True))
        ref, _ = QO.forward(cfg, P, ids, oc)
        assert rel(got, ref[:, -1:]) <= REL


def test_layer_call_matches_deferred_residual(models):
    """Layer.__call__ (separate residual add, as engine/model.py:313-316 writes it) and the
    model's deferred add (inside the next rms_norm) give the same bits."""
    cfg, model, P = models
    from qvex import glue
    x = (torch.randn((1, 3, cfg.hidden_size), device="cuda")).to(torch.bfloat16)
    layer = model.layers[0]
    a = layer(x, model.make_cache()[0])
    h, mo = layer.forward_deferred(x, None, model.make_cache()[0])
    assert torch.equal(a.view(torch.int16), glue.add(h, mo).view(torch.int16))


def test_graph_decode_matches_eager_greedy(models):
    """DecodeGraph (one CUDA graph per step, position and tokens on the device, states
    updated in place) picks the same tokens as eager greedy decoding, bit for bit."""
    cfg, model, P = models
    from qvex.qwen35 import DecodeGraph
    from qvex.sampler import sample_pick, sample_scores
    rng = np.random.default_rng(2)
    B, L, n = 2, 12, 6
    ids = torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, L)).astype(np.int32)).cuda()

    cache = model.make_cache(capacity=64)
    logits = model(ids, cache, last_only=True)
    tok = sample_pick(sample_scores(logits.view(B, -1), temperature=0.0), True).view(B, 1)
    eager = []
    for _ in range(n):
        logits = model(tok, cache, last_only=True)
        tok = sample_pick(sample_scores(logits.view(B, -1), temperature=0.0), True).view(B, 1)
        eager.append(tok.view(-1).clone())
    eager = torch.stack(eager)

    cache = model.make_cache(capacity=64)
    logits = model(ids, cache, last_only=True)
    first = sample_pick(sample_scores(logits.view(B, -1), temperature=0.0), True).view(B, 1)
    g = DecodeGraph(model, cache, first, pos=L)
    got = g.run(n)
    assert torch.equal(got, eager), (got, eager)
    assert all(c.offset == L + n for c in cache)


def test_loaded_checkpoints_give_the_same_logits(tmp_path):
    """A model loaded from an MLX-layout checkpoint directory (qvex.checkpoint.load_model) and
    from the native .q35 file (load_q35) computes exactly the logits of the same parameters
    built in memory."""
    from qvex.checkpoint import load_model, load_q35, save_checkpoint, write_q35
    from qvex.qwen35 import Qwen35, random_params
    cfg = small_cfg()
    P = random_params(cfg, 17, "cpu")
    save_checkpoint(tmp_path / "mlx", cfg, P)
    write_q35(tmp_path / "m.q35", cfg, P)
    ids = torch.randint(0, cfg.vocab_size, (2, 9), device="cuda", dtype=torch.int32)
    ref = Qwen35.from_params(cfg, {k: v.cuda() for k, v in P.items()})
    want = host(ref(ids, ref.make_cache(), last_only=False))
    for m in (load_model(tmp_path / "mlx"), load_q35(tmp_path / "m.q35")):
        assert np.array_equal(host(m(ids, m.make_cache(), last_only=False)), want)
