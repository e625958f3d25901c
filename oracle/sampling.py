"""Oracle: sampling and speculative verification (test infrastructure only).

Restates vllmlite/sampling.py:16-64 and vllmlite/speculative.py:86-100.
"""

from __future__ import annotations

import numpy as np


def penalize(logits: np.ndarray, seen, penalty: float) -> None:
    """Repetition penalty on every distinct seen token: positive logits divided,
    non-positive multiplied. Follows vllmlite/sampling.py:8-13."""
    if penalty == 1.0 or len(seen) == 0:
        return
    idx = np.unique(np.asarray(seen, np.int64))
    cur = logits[idx]
    logits[idx] = np.where(cur > 0, cur / penalty, cur * penalty)


def top_k_mask(logits: np.ndarray, k: int) -> None:
    """Keep logits >= the k-th largest. Follows vllmlite/sampling.py:16-20."""
    if 0 < k < logits.size:
        kth = np.sort(logits)[-k]
        logits[logits < kth] = -np.inf


def top_p_keep(logits: np.ndarray, p: float) -> np.ndarray:
    """Boolean keep-mask of the nucleus: tokens in descending-logit order are kept
    while the probability mass before them is < p (the crossing token is kept).
    Follows vllmlite/sampling.py:23-33 (stable order of np.argsort(-logits))."""
    if p >= 1.0:
        return np.ones(logits.size, bool)
    order = np.argsort(-logits, kind="quicksort")
    z = logits[order] - logits[order].max()
    probs = np.exp(z)
    probs = probs / probs.sum()
    before = np.cumsum(probs) - probs
    keep = np.zeros(logits.size, bool)
    keep[order[before < p]] = True
    return keep


def greedy(logits: np.ndarray, eos_id=None, num_generated=0, min_tokens=0, seen=(),
           penalty=1.0) -> int:
    """The greedy path of vllmlite/sampling.py:41-57: EOS masked until
    min_tokens, repetition penalty, then the FIRST index of the maximum."""
    x = logits.astype(np.float32, copy=True)
    if eos_id is not None and num_generated < min_tokens:
        x[eos_id] = -np.inf
    penalize(x, seen, penalty)
    return int(np.argmax(x))


def softmax(x: np.ndarray) -> np.ndarray:
    """float32 softmax with the max subtracted. Follows vllmlite/sampling.py:35-38."""
    z = x - x.max()
    e = np.exp(z)
    return e / e.sum()


def sample_with_uniform(logits: np.ndarray, temperature: float, top_k: int, top_p: float, u: float,
                        eos_id=None, num_generated=0, min_tokens=0, seen=(), penalty=1.0):
    """The temperature branch of vllmlite/sampling.py:41-64 with the draw made
    from a given uniform: EOS masked until min_tokens (:51-52), repetition
    penalty (:54), division by the temperature (:59), top-k (:60), top-p
    (:61), softmax (:63), then numpy's Generator.choice(size, p=probs) (:64),
    which takes one rng.random() double u and returns the first index whose
    float64 CDF (cumsum of probs divided by its last value) exceeds u.
    Returns (token, keep mask, probs float32)."""
    x = logits.astype(np.float32, copy=True)
    if eos_id is not None and num_generated < min_tokens:
        x[eos_id] = -np.inf
    penalize(x, seen, penalty)
    x /= np.float32(temperature)
    top_k_mask(x, top_k)
    x[~top_p_keep(x, top_p)] = -np.inf
    probs = softmax(x)
    cdf = np.cumsum(probs.astype(np.float64))
    cdf /= cdf[-1]
    tok = int(np.searchsorted(cdf, u, side="right"))
    return tok, np.isfinite(x), probs


def verify(logits: np.ndarray, drafts) -> tuple[list[int], int]:
    """Greedy speculative acceptance. Follows vllmlite/speculative.py:86-100:
    accept drafts while each equals the row's argmax; the first mismatch emits
    the model's token; if all are accepted the last row adds a bonus token."""
    out = []
    for i, d in enumerate(drafts):
        t = int(np.argmax(logits[i]))
        out.append(t)
        if t != d:
            return out, i
    out.append(int(np.argmax(logits[len(drafts)])))
    return out, len(drafts)
