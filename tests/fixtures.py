"""Golden-fixture readers shared by the CPU and GPU suites."""

from __future__ import annotations

import json
import os
from types import SimpleNamespace

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

TINY = dict(n_layers=2, n_heads=4, n_kv_heads=2, d_model=64, d_ff=128, max_seq_len=512)
BENCH = dict(n_layers=6, n_heads=8, n_kv_heads=4, d_model=384, d_ff=1024, max_seq_len=512)

PROMPTS = [
    "paged attention keeps every sequence in fixed size blocks",
    "z",
    "continuous batching rebuilds the batch on every single forward pass, so",
    "kv",
    "a block table maps logical positions to physical cache blocks",
]
REPEATS = [
    "red green blue red green blue red green blue red green blue red green blue",
    "0123456789 0123456789 0123456789 0123456789 0123456789 0123456789",
]


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def weights_manifest():
    with open(os.path.join(GOLDEN, "weights.json")) as f:
        return json.load(f)


def attention_cases():
    """Yield (case index, inputs, expected) for every golden attention case."""
    z = load("attention.npz")
    for i, (seed, q_len, H, KV, D, bs, ctx) in enumerate(z["cases"]):
        rng = np.random.default_rng(int(seed))
        nb = (ctx + bs - 1) // bs
        total = nb + 5
        ck = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
        cv = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
        bids = [int(b) for b in rng.permutation(total)[:nb]]
        q = rng.standard_normal((q_len, H, D)).astype(np.float32)
        yield i, dict(q=q, cache_k=ck, cache_v=cv, block_ids=bids, block_size=int(bs), ctx=int(ctx),
                      n_kv=int(KV), scale=1.0 / np.sqrt(D), insha=z[f"insha_{i}"]), z[f"out_{i}"]


def replay_steps(name):
    """Step records of a golden replay: list of (seqs, cow, logits)."""
    z = load(name)
    steps = []
    sr = z["seq_rows"]
    for si, row0, nrows in z["step_meta"]:
        seqs = []
        for r in sr[sr[:, 0] == si]:
            _, start, n, count, to, tn, bo, bn, do, dn = (int(v) for v in r)
            seqs.append(dict(start=start, n=n, count=count, tokens=z["tokens"][to:to + tn].tolist(),
                             block_ids=z["block_ids"][bo:bo + bn].tolist(),
                             drafts=z["drafts"][do:do + dn].tolist()))
        cow = [(int(a), int(b)) for s, a, b in z["cow"] if s == si]
        steps.append((seqs, cow, z["logits"][row0:row0 + nrows]))
    return steps


def as_scheduler_output(seqs, cow=()):
    """A duck-typed SchedulerOutput (vllmlite/scheduler.py:22-49) for a step
    record: what ModelRunner.execute reads and nothing else."""
    items = []
    for s in seqs:
        # token_ids only needs to hold the pushed tokens at their positions
        toks = [0] * s["start"] + list(s["tokens"])
        seq = SimpleNamespace(token_ids=toks, draft_token_ids=list(s["drafts"]),
                              table=SimpleNamespace(block_ids=list(s["block_ids"])))
        items.append(SimpleNamespace(seq=seq, start_pos=s["start"], num_tokens=s["n"]))
    return SimpleNamespace(scheduled=items, cow=list(cow))


def streams(name, key=""):
    z = load(name)
    lens = z[f"{key}lens"]
    toks = z[f"{key}tokens"].astype(np.int64)
    out, o = [], 0
    for n in lens:
        out.append(toks[o:o + n].tolist())
        o += n
    return out
