"""Speculative decoding with the model's multi-token-prediction (MTP) head, on libqvex.

Mirrors engine/mtp.py and engine/speculative.py:

* ``MTPHead`` (engine/mtp.py:19-82): given the main model's hidden state at position i and
  the token at i+1 it predicts token i+2 --
  x = fc([rms(embed(tok)), rms(h)]) -> one gated-attention + MLP block -> norm -> lm_head,
  sharing the main model's embedding and lm_head; its attention keeps its own KV cache.
* ``mtp_prefill`` (engine/speculative.py:26-41) feeds the head the (h_i, tok_{i+1}) pairs of
  a prefill chunk.
* ``decode`` (engine/speculative.py:44-118) yields tokens: plain steps, or MTP cycles that
  draft one token, verify [last, draft] in one 2-token pass of the main model with
  keep_prev (the M = 2 decode projections, the recurrence's pre-last-step snapshot), and
  accept it (greedy: the draft equals the argmax; sampling: with probability p(draft)) or
  roll every cache back one token and emit a token drawn from the residual distribution.

Random numbers: the acceptance test draws from a seeded host generator and the token draws
from the sampler's counter-based device generator, so runs are reproducible; they agree
with the reference's mx.random streams in distribution, not draw for draw.
"""
from __future__ import annotations

from typing import Callable, Iterator

import numpy as np
import torch

from . import glue
from .checkpoint import read_safetensors
from .model import QLinear
from .qwen35 import KVCache, Layer, Qwen35
from .sampler import Sampler, sample_pick

MAX_PENDING = 1024  # beyond this, the MTP head misses the oldest positions (engine/speculative.py:23)


class MTPHead:
    """The multi-token-prediction head (engine/mtp.py:19-82)."""

    def __init__(self, model: Qwen35, w: dict, group_size: int = 64, bits: int = 4, hidden_mode: str = "pre"):
        cfg = model.cfg
        self.model = model
        self.eps = cfg.rms_norm_eps
        self.hidden_mode = hidden_mode  # "pre": raw last-layer output, "post": after the final norm

        def qlin(prefix):
            return QLinear(w[f"{prefix}.weight"], w[f"{prefix}.scales"], w[f"{prefix}.biases"], group_size, bits)

        self.fc = qlin("mtp.fc")
        self.norm_emb = w["mtp.pre_fc_norm_embedding.weight"]
        self.norm_hid = w["mtp.pre_fc_norm_hidden.weight"]
        self.norm_out = w["mtp.norm.weight"]
        sa = "mtp.layers.0.self_attn"
        p = {"input_layernorm": w["mtp.layers.0.input_layernorm.weight"],
             "post_attention_layernorm": w["mtp.layers.0.post_attention_layernorm.weight"],
             "self_attn": {**{n: qlin(f"{sa}.{n}") for n in ("q_proj", "k_proj", "v_proj", "o_proj")},
                           "q_norm": w[f"{sa}.q_norm.weight"], "k_norm": w[f"{sa}.k_norm.weight"]},
             "mlp": {n: qlin(f"mtp.layers.0.mlp.{n}") for n in ("gate_proj", "up_proj", "down_proj")}}
        # the same block as a main full-attention layer (index of one such layer)
        self.layer = Layer(cfg, cfg.full_attention_interval - 1, p)

    def make_cache(self) -> KVCache:
        return KVCache()

    def __call__(self, hidden: torch.Tensor, next_ids: torch.Tensor, cache: KVCache, last_only: bool = True):
        """hidden [B, T, H] (main model, pre-norm), next_ids [B, T] -> logits [B, 1 or T, V]."""
        if self.hidden_mode == "post":
            hidden = glue.rms_norm(hidden, self.model.norm, self.eps)
        e = glue.rms_norm(self.model.embed(next_ids), self.norm_emb, self.eps)
        h = glue.rms_norm(hidden.contiguous(), self.norm_hid, self.eps)
        x = self.fc(torch.cat([e, h], dim=-1))
        x = self.layer(x, cache)
        if last_only:
            x = x[:, -1:, :].contiguous()
        return self.model.lm_head(glue.rms_norm(x, self.norm_out, self.eps))


def mtp_param_names(cfg) -> dict[str, tuple[int, int] | tuple[int]]:
    """Shapes of the MTP head's tensors ((N, K) for quantized modules, (n,) for norms)."""
    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    sa, ml = "mtp.layers.0.self_attn", "mtp.layers.0.mlp"
    return {"mtp.fc": (H, 2 * H), f"{sa}.q_proj": (2 * Hq * D, H), f"{sa}.k_proj": (Hkv * D, H),
            f"{sa}.v_proj": (Hkv * D, H), f"{sa}.o_proj": (H, Hq * D), f"{ml}.gate_proj": (I, H),
            f"{ml}.up_proj": (I, H), f"{ml}.down_proj": (H, I),
            "mtp.pre_fc_norm_embedding.weight": (H,), "mtp.pre_fc_norm_hidden.weight": (H,), "mtp.norm.weight": (H,),
            "mtp.layers.0.input_layernorm.weight": (H,), "mtp.layers.0.post_attention_layernorm.weight": (H,),
            f"{sa}.q_norm.weight": (D,), f"{sa}.k_norm.weight": (D,)}


def random_mtp_params(cfg, seed: int, device) -> dict:
    """Random MTP weights of the head's shapes (synthetic 4-bit g64, as the main model's)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = {}
    for name, shape in mtp_param_names(cfg).items():
        if len(shape) == 1:
            w[name] = (1.0 + 0.05 * torch.randn(shape[0], device=device, generator=g)).to(torch.bfloat16)
            continue
        N, K = shape
        s = (torch.randn((N, K // 64), device=device, generator=g).abs() * 0.002).to(torch.bfloat16)
        w[f"{name}.weight"] = torch.randint(-2 ** 31, 2 ** 31, (N, K // 8), dtype=torch.int64, device=device,
                                            generator=g).to(torch.int32)
        w[f"{name}.scales"] = s
        w[f"{name}.biases"] = (-8.0 * s.float()).to(torch.bfloat16)
    return w


def load_mtp(model: Qwen35, path, hidden_mode: str = "pre", device="cuda") -> MTPHead:
    """engine/mtp.py:85-87: the head from a safetensors file with group_size / bits metadata."""
    w, meta = read_safetensors(path)
    w = {k: v.to(torch.device(device)) for k, v in w.items()}
    return MTPHead(model, w, int(meta.get("group_size", 64)), int(meta.get("bits", 4)), hidden_mode)


def mtp_prefill(mtp: MTPHead, mtp_cache: KVCache, hidden: torch.Tensor, ids: torch.Tensor,
                prev_hidden: torch.Tensor | None):
    """engine/speculative.py:26-41: feed the head the (h_i, tok_{i+1}) pairs of a chunk;
    returns the hidden of the chunk's last token (the next chunk's prev_hidden)."""
    if prev_hidden is not None:
        h_in, next_ids = torch.cat([prev_hidden, hidden[:, :-1]], dim=1), ids
    else:
        h_in, next_ids = hidden[:, :-1], ids[:, 1:]
    if next_ids.shape[1] > 0:
        mtp(h_in.contiguous(), next_ids.contiguous(), mtp_cache)
    return hidden[:, -1:]


def decode(model: Qwen35, sampler: Sampler, cache, first_logits: torch.Tensor, last_hidden=None,
           mtp: MTPHead | None = None, mtp_cache: KVCache | None = None,
           use_mtp: Callable[[], bool] = lambda: True, stats: dict | None = None,
           forced: list[int] | None = None, seed: int = 0) -> Iterator[int]:
    """Generator of token ids (engine/speculative.py:44-118).  ``stats`` gets 'cycles' /
    'accepted' (MTP) and 'plain' counters; ``forced`` tokens are emitted next, in order, on
    plain steps."""
    forced = forced if forced is not None else []
    stats = stats if stats is not None else {}
    for k in ("cycles", "accepted", "plain"):
        stats.setdefault(k, 0)
    rng = np.random.default_rng(seed)
    V = model.cfg.vocab_size
    dev = first_logits.device

    feed = sampler.pick(sampler.scores(first_logits.reshape(1, V))).reshape(())
    sampler.observe(feed)
    pend_h = [last_hidden] if mtp is not None else []
    pend_ids = [feed.reshape(1, 1)] if mtp is not None else []
    yield int(feed)

    while True:
        if mtp is not None and pend_h and not forced and use_mtp():
            h_in = pend_h[0] if len(pend_h) == 1 else torch.cat(pend_h, dim=1)
            id_in = pend_ids[0] if len(pend_ids) == 1 else torch.cat(pend_ids, dim=1)
            draft = mtp(h_in.contiguous(), id_in.to(torch.int32).contiguous(), mtp_cache)[0, -1].float().argmax()
            ids = torch.stack([feed.reshape(()), draft.to(feed.dtype)]).reshape(1, 2).to(torch.int32)
            logits, hidden = model(ids, cache, last_only=False, return_hidden=True, keep_prev=True)

            s0 = sampler.scores(logits[0, 0:1]).reshape(V)
            if sampler.greedy:
                resample = s0.argmax()
                accept = bool(resample == draft)
            else:
                accept = bool(rng.random() < float(torch.exp(s0[draft])))
                masked = s0.clone()
                masked[draft] = -float("inf")
                sampler._draws += 1
                resample = sample_pick(masked.reshape(1, V), False, sampler._seed, sampler._draws).reshape(())
            t1 = sampler.pick(sampler.scores(logits[0, 1:2], extra_seen=draft.reshape(1))).reshape(())
            stats["cycles"] += 1

            if accept:
                stats["accepted"] += 1
                sampler.observe(draft)
                sampler.observe(t1)
                for c in cache:
                    if hasattr(c, "ssm_prev"):
                        c.conv_prev = c.ssm_prev = None
                pend_h = [hidden]
                pend_ids = [torch.stack([draft.to(t1.dtype), t1]).reshape(1, 2)]
                feed = t1
                yield int(draft)
                yield int(t1)
            else:
                for c in cache:
                    c.rollback(1)
                sampler.observe(resample)
                pend_h, pend_ids, feed = [hidden[:, :1]], [resample.reshape(1, 1)], resample
                yield int(resample)
        else:
            tok_in = feed.reshape(1, 1).to(torch.int32)
            if mtp is not None:
                logits, hidden = model(tok_in, cache, return_hidden=True)
            else:
                logits, hidden = model(tok_in, cache), None
            t = (torch.tensor(forced.pop(0), device=dev) if forced
                 else sampler.pick(sampler.scores(logits.reshape(1, V))).reshape(()))
            sampler.observe(t)
            stats["plain"] += 1
            if mtp is not None:
                pend_h.append(hidden)
                pend_ids.append(t.reshape(1, 1))
                if len(pend_h) > MAX_PENDING:
                    pend_h, pend_ids = pend_h[-MAX_PENDING:], pend_ids[-MAX_PENDING:]
            feed = t
            yield int(t)
