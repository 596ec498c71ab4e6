"""The C restatement of Sampler.scores (orc_sample_scores) against a second, independent
transcription of engine/sampler.py:30-62 in numpy, op for op (argpartition, sort,
softmax, cumsum - probs < top_p, where, logsumexp; fp32 throughout).  MLX itself is not
installed, so this pins the oracle to the reference's algorithm rather than to MLX's
rounding.  CPU only.
"""
import numpy as np
import pytest

import detrand
import oracle as O


def scores_numpy(logits, seen, temperature, top_p, top_k, presence_penalty):
    """engine/sampler.py Sampler.scores for one row, numpy in place of mlx.core."""
    logits = logits.astype(np.float32)
    if seen is not None and presence_penalty:
        logits = logits - np.float32(presence_penalty) * seen
    if temperature <= 0:
        return logits
    logits = logits / np.float32(temperature)
    V = logits.shape[-1]
    if 0 < top_k < V:
        cand = logits[np.argpartition(-logits, top_k - 1)[:top_k]]
    else:
        cand = logits
    cand = np.sort(cand)[::-1]
    cutoff = cand[-1]
    if 0 < top_p < 1:
        e = np.exp(cand - cand.max())
        probs = (e / e.sum(dtype=np.float32)).astype(np.float32)
        keep = (np.cumsum(probs, dtype=np.float32) - probs) < np.float32(top_p)
        cutoff = np.min(np.where(keep, cand, np.float32(np.inf)))
    logits = np.where(logits >= cutoff, logits, np.float32(-np.inf))
    m = logits.max()
    lse = m + np.log(np.exp(logits - m).sum(dtype=np.float32))
    return (logits - lse).astype(np.float32)


@pytest.mark.parametrize("V,T,top_p,top_k,pp", [
    (248320, 0.6, 0.95, 20, 0.0),
    (5000, 1.0, 0.5, 64, 0.0),
    (3000, 0.7, 0.9, 1, 0.0),
    (4000, 0.8, 1.0, 100, 0.0),
    (2000, 1.2, 0.0, 0, 0.0),
    (6000, 0.6, 0.95, 20, 1.5),
    (500, 0.0, 0.95, 20, 0.5),
])
def test_oracle_matches_numpy_transcription(V, T, top_p, top_k, pp):
    x = (detrand.normal((1, V), V + top_k) * 3).astype(np.float32)
    seen = None
    if pp:
        seen = np.zeros(V, np.float32)
        seen[detrand.integers((V // 10,), V, V)] = 1.0
    ref = scores_numpy(x[0], seen, T, top_p, top_k, pp)
    got = O.sample_scores(x, seen, T, top_p, top_k, pp)[0]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    # numpy sums pairwise, the oracle in index order: a few ulps of scores near -10
    assert np.max(np.abs(got[fin] - ref[fin])) <= 1e-5
