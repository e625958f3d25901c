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
