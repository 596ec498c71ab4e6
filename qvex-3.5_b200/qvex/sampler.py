"""Token sampling after the lm_head projection, mirroring engine/sampler.py.

``SamplingParams`` and ``Sampler`` keep the reference's fields and methods:
``scores(logits, extra_seen)`` builds full-vocabulary scores (penalised logits when
greedy, filtered log-probabilities when sampling, engine/sampler.py:30-62) and
``pick(scores)`` draws a token (argmax, or a draw from softmax(scores):
engine/sampler.py:63-64); ``observe(tok)`` marks a token as seen for the presence penalty.
Both run in libqvex.so (qvx_sample_scores / qvx_sample_pick) on the current stream and
stay on the device: no host sync per token.  Draws come from a counter-based generator
keyed by the seed and a per-call counter, so they agree with the reference's
mx.random.categorical in distribution, not draw for draw.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from ._lib import _P, check, lib
from .core import _ptr, _require_cuda, _stream


@dataclass
class SamplingParams:
    temperature: float = 0.6
    top_p: float = 0.95
    top_k: int = 20
    presence_penalty: float = 0.0
    max_tokens: int = 2048
    seed: int | None = None


def sample_scores(logits: torch.Tensor, temperature: float = 0.6, top_p: float = 0.95, top_k: int = 20,
                  presence_penalty: float = 0.0, seen: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 scores [..., V] of bf16 or fp32 logits [..., V] (Sampler.scores)."""
    _require_cuda("logits", logits, (torch.bfloat16, torch.float32))
    V = logits.shape[-1]
    x = logits.reshape(-1, V).contiguous()
    if seen is not None:
        _require_cuda("seen", seen, (torch.float32,))
        if seen.numel() != V:
            raise ValueError(f"seen has {seen.numel()} entries for a vocabulary of {V}")
        seen = seen.contiguous()
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    check(lib().qvx_sample_scores(_ptr(x), 0 if x.dtype == torch.bfloat16 else 1, _ptr(seen), _ptr(out),
                                  x.shape[0], V, float(temperature), float(top_p), int(top_k),
                                  float(presence_penalty), _stream(x)), "qvx_sample_scores")
    return out.reshape(logits.shape)


def sample_pick(scores: torch.Tensor, greedy: bool, seed: int = 0, offset: int = 0, *,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """int32 tokens [...] from fp32 scores [..., V] (Sampler.pick); ``out`` (contiguous int32,
    one element per row) receives them when given."""
    _require_cuda("scores", scores, (torch.float32,))
    V = scores.shape[-1]
    s = scores.reshape(-1, V).contiguous()
    if out is not None:
        if out.dtype != torch.int32 or out.numel() != s.shape[0] or not out.is_contiguous():
            raise ValueError("out must be a contiguous int32 tensor with one element per row")
        tok = out.view(-1)
    else:
        tok = torch.empty(s.shape[0], dtype=torch.int32, device=s.device)
    check(lib().qvx_sample_pick(_ptr(s), _ptr(tok), s.shape[0], V, 1 if greedy else 0, seed & (2**64 - 1),
                                offset & (2**64 - 1), _stream(s)), "qvx_sample_pick")
    return out if out is not None else tok.reshape(scores.shape[:-1])


class Sampler:
    """engine/sampler.py's Sampler on the GPU: same constructor, ``greedy``, ``scores``,
    ``pick`` and ``observe``."""

    def __init__(self, params: SamplingParams, vocab_size: int, device=None):
        self.p = params
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        # presence mask, updated on the device: no host sync per token
        self.seen = torch.zeros(vocab_size, dtype=torch.float32, device=dev) if params.presence_penalty else None
        self._seed = params.seed if params.seed is not None else int.from_bytes(os.urandom(8), "little")
        self._draws = 0

    @property
    def greedy(self) -> bool:
        return self.p.temperature <= 0

    def scores(self, logits: torch.Tensor, extra_seen: torch.Tensor | None = None) -> torch.Tensor:
        """Scores over the whole vocabulary: the logits minus the presence penalty when greedy,
        else log-probabilities restricted to the top-k / top-p set."""
        p = self.p
        seen = self.seen
        if seen is not None and extra_seen is not None:
            seen = seen.clone()
            seen[extra_seen.long()] = 1.0
        return sample_scores(logits, p.temperature, p.top_p, p.top_k, p.presence_penalty, seen)

    def pick(self, scores: torch.Tensor) -> torch.Tensor:
        if self.greedy:
            return sample_pick(scores, True)
        self._draws += 1
        return sample_pick(scores, False, self._seed, self._draws)

    def observe(self, tok) -> None:
        if self.seen is not None:
            idx = tok.long() if torch.is_tensor(tok) else torch.as_tensor(tok, device=self.seen.device).long()
            self.seen[idx] = 1.0
