"""Speculative decoding with the MTP head (qvex.speculative, engine/speculative.py) on a small
random-initialised Qwen3.5-shaped model.

With a greedy sampler, speculative decoding must emit the plain greedy sequence: a cycle
verifies [last, draft] in one 2-token pass with keep_prev, accepts the draft only when it is
the argmax, and otherwise rolls every cache back one token (the DeltaNet states to their
pre-last-step snapshots, the KV caches' offsets) and emits the argmax.  Two drafters:
  * the real MTP head with random weights (its drafts are mostly wrong: the rollback path);
  * a stand-in that drafts the plain sequence's next token on two calls of three and a wrong
    token on the third, so both the accept and the rollback paths run many times.
The verify pass runs the M = 2 kernels and the plain steps the M = 1 kernels, whose fp32
sums differ in the last bits; so where the two sequences part, the plain step's two
candidate logits must be a tie of bf16 values (within one ulp), else the test fails."""
import numpy as np
import pytest
import torch

from test_model_oracle import small_cfg

pytestmark = pytest.mark.gpu

N_TOKENS = 24


@pytest.fixture(scope="module")
def setup():
    from qvex.qwen35 import Qwen35, random_params
    cfg = small_cfg()
    model = Qwen35.from_params(cfg, random_params(cfg, 23, "cuda"))
    return cfg, model


def plain_run(cfg, model, prompt, n):
    """Plain greedy decode; returns the tokens and every step's logits."""
    from qvex.sampler import Sampler, SamplingParams
    from qvex.speculative import decode
    sampler = Sampler(SamplingParams(temperature=0.0), cfg.vocab_size)
    cache = model.make_cache()
    first = model(prompt, cache, last_only=True)
    toks = []
    for t in decode(model, sampler, cache, first):
        toks.append(t)
        if len(toks) == n:
            break
    # logits each plain step saw (recomputed with a fresh cache, one token at a time)
    cache2 = model.make_cache()
    logits = [model(prompt, cache2, last_only=True).float().reshape(-1)]
    for t in toks[:-1]:
        logits.append(model(torch.tensor([[t]], dtype=torch.int32, device="cuda"), cache2).float().reshape(-1))
    return toks, logits


def agree_up_to_ties(plain, plain_logits, spec):
    for i, (a, b) in enumerate(zip(plain, spec)):
        if a != b:
            lg = plain_logits[i]
            gap = float(lg[a] - lg[b])
            ulp = float(abs(lg[a])) * 2 ** -7 + 1e-6
            assert abs(gap) <= ulp, f"token {i}: {a} vs {b}, logit gap {gap} (not a tie)"
            return i
    return len(plain)


class OracleDrafter:
    """Drafts the plain sequence's next token, except on every third call (a wrong token)."""

    def __init__(self, plain, vocab, emitted):
        self.plain, self.vocab, self.emitted, self.calls = plain, vocab, emitted, 0

    def __call__(self, hidden, next_ids, cache, last_only=True):
        self.calls += 1
        i = min(self.emitted[0], len(self.plain) - 1)
        tok = self.plain[i] if self.calls % 3 else (self.plain[i] + 1) % self.vocab
        out = torch.full((1, 1, self.vocab), -10.0, dtype=torch.bfloat16, device="cuda")
        out[0, 0, tok] = 10.0
        return out


@pytest.mark.parametrize("drafter", ["mtp_head", "oracle"])
def test_greedy_speculative_equals_plain(setup, drafter):
    from qvex.sampler import Sampler, SamplingParams
    from qvex.speculative import MTPHead, decode, mtp_prefill, random_mtp_params
    cfg, model = setup
    prompt = torch.randint(0, cfg.vocab_size, (1, 13), device="cuda", dtype=torch.int32,
                           generator=torch.Generator(device="cuda").manual_seed(4))
    plain, plain_logits = plain_run(cfg, model, prompt, N_TOKENS)

    sampler = Sampler(SamplingParams(temperature=0.0), cfg.vocab_size)
    cache = model.make_cache()
    first, hidden = model(prompt, cache, last_only=True, return_hidden=True)
    emitted = [0]
    if drafter == "mtp_head":
        mtp = MTPHead(model, random_mtp_params(cfg, 2, "cuda"))
        mtp_cache = mtp.make_cache()
        last = mtp_prefill(mtp, mtp_cache, hidden, prompt, None)
    else:
        mtp = OracleDrafter(plain, cfg.vocab_size, emitted)
        mtp_cache = None
        last = hidden[:, -1:]
    stats = {}
    spec = []
    for t in decode(model, sampler, cache, first, last, mtp=mtp, mtp_cache=mtp_cache, stats=stats):
        spec.append(t)
        emitted[0] = len(spec)
        if len(spec) >= N_TOKENS:
            break
    n = agree_up_to_ties(plain, plain_logits, spec[:N_TOKENS])
    assert stats["cycles"] > 0
    if drafter == "oracle":
        assert stats["accepted"] > 0 and stats["accepted"] < stats["cycles"], stats
        assert n >= 8, f"sequences parted at token {n} (a tie), too early to have tested the cycles"
    print(drafter, stats, "agreed on", n, "tokens")


def test_plain_steps_and_forced_tokens(setup):
    """use_mtp() False runs plain steps; forced tokens are emitted next, in order."""
    from qvex.sampler import Sampler, SamplingParams
    from qvex.speculative import decode
    cfg, model = setup
    prompt = torch.randint(0, cfg.vocab_size, (1, 5), device="cuda", dtype=torch.int32)
    sampler = Sampler(SamplingParams(temperature=0.0), cfg.vocab_size)
    cache = model.make_cache()
    first = model(prompt, cache)
    forced = []
    out, stats = [], {}
    for t in decode(model, sampler, cache, first, forced=forced, stats=stats):
        out.append(t)
        if len(out) == 2:
            forced += [7, 9]
        if len(out) == 6:
            break
    assert out[2:4] == [7, 9] and stats["plain"] == 5 and stats["cycles"] == 0


def test_sampling_speculative_runs(setup):
    """Non-greedy cycles (acceptance with probability p(draft), residual draws) run and keep
    the caches consistent: the sequence continues without error and offsets match."""
    from qvex.sampler import Sampler, SamplingParams
    from qvex.speculative import MTPHead, decode, mtp_prefill, random_mtp_params
    cfg, model = setup
    prompt = torch.randint(0, cfg.vocab_size, (1, 7), device="cuda", dtype=torch.int32)
    sampler = Sampler(SamplingParams(temperature=0.8, top_p=0.95, top_k=20, seed=3), cfg.vocab_size)
    cache = model.make_cache()
    first, hidden = model(prompt, cache, last_only=True, return_hidden=True)
    mtp = MTPHead(model, random_mtp_params(cfg, 5, "cuda"))
    mc = mtp.make_cache()
    last = mtp_prefill(mtp, mc, hidden, prompt, None)
    out, stats = [], {}
    for t in decode(model, sampler, cache, first, last, mtp=mtp, mtp_cache=mc, stats=stats):
        out.append(t)
        if len(out) >= 12:
            break
    assert all(0 <= t < cfg.vocab_size for t in out) and stats["cycles"] > 0
    # every cache saw the prompt and every emitted token but the newest (or, stopped between
    # the two tokens of an accepted cycle, the newest too)
    assert all(c.offset in (7 + len(out) - 1, 7 + len(out)) for c in cache), [c.offset for c in cache]
    assert len({c.offset for c in cache}) == 1
