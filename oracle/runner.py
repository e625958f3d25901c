"""Oracle: ModelRunner.execute flatten and copy-on-write (test infrastructure only).

Restates vllmlite/runner.py:35-100 of the reference on plain step records, so
a replayed schedule (tests/golden/*.npz) can be pushed through the oracle
without the reference's Scheduler.
"""

from __future__ import annotations

import numpy as np

from .attention import table_slots
from .model import Shape, forward


def flatten(steps_seqs, block_size: int):
    """Build (token_ids, positions, seq_meta, last_idx, rows) for one pass.

    steps_seqs: list of dicts with keys start, n, count, block_ids, tokens
    (tokens = the n token ids at positions start..start+n-1). Follows
    vllmlite/runner.py:66-90: positions start..start+n-1, read slots for
    0..start+n-1 through the block table, write slots = read_slots[start:],
    and logit rows for the last `count` tokens of each sequence.
    """
    token_ids, positions, seq_meta, last_idx, rows = [], [], [], [], []
    for s in steps_seqs:
        start, n, count = s["start"], s["n"], s["count"]
        off = len(token_ids)
        token_ids += list(s["tokens"])
        positions += range(start, start + n)
        rslots = table_slots(s["block_ids"], block_size, start + n)
        seq_meta.append((off, n, rslots[start:], rslots))
        rows.append((len(last_idx), count))
        last_idx += range(off + n - count, off + n)
    return (np.asarray(token_ids, np.int64), np.asarray(positions, np.int64), seq_meta,
            np.asarray(last_idx, np.int64), rows)


def copy_blocks(cache_k, cache_v, pairs, block_size: int) -> None:
    """Copy whole blocks src -> dst in every layer, K and V.

    Follows vllmlite/runner.py:54-60; cache_* are [L, slots, n_kv, D].
    """
    for src, dst in pairs:
        s = slice(src * block_size, (src + 1) * block_size)
        d = slice(dst * block_size, (dst + 1) * block_size)
        cache_k[:, d] = cache_k[:, s]
        cache_v[:, d] = cache_v[:, s]


class OracleRunner:
    """Replays step records through the NumPy forward with its own KV cache."""

    def __init__(self, cfg: Shape, weights, num_blocks: int, block_size: int, dtype=np.float32):
        self.cfg, self.w, self.bs, self.dtype = cfg, weights, block_size, dtype
        shape = (cfg.n_layers, num_blocks * block_size, cfg.n_kv_heads, cfg.head_dim)
        self.cache_k = np.zeros(shape, dtype)
        self.cache_v = np.zeros(shape, dtype)

    def execute(self, seqs, cow=()):
        if cow:
            copy_blocks(self.cache_k, self.cache_v, cow, self.bs)
        tok, pos, meta, last, rows = flatten(seqs, self.bs)
        logits = forward(self.cfg, self.w, tok, pos, self.cache_k, self.cache_v, meta, last,
                         dtype=self.dtype)
        return logits, rows
