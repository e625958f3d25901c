"""CPU: the oracle (oracle/) is pinned to the reference's own outputs.

Every fixture under tests/golden/ was produced by the reference itself
(tests/golden/make_golden.py). Before any GPU result is compared with the
oracle, the oracle must reproduce those fixtures.
"""

import hashlib

import numpy as np
import pytest

from oracle import attention as A
from oracle import model as M
from oracle import runner as R
from oracle import sampling as SP
from tests import fixtures as F


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["tiny", "bench"])
def test_seeded_weights_are_bit_identical(name):
    man = F.weights_manifest()[name]
    cfg = M.Shape(vocab_size=261, **man["shape"])
    w = M.seeded_weights(cfg)
    assert {k: sha(v) for k, v in w.items()} == man["sha256"]


def test_rope_tables_bit_identical():
    z = F.load("rope.npz")
    for key in z.files:
        if key.startswith("cos_"):
            _, D, P = key.split("_")
            c, s = A.rope_tables(int(D), int(P))
            np.testing.assert_array_equal(c, z[key])
            np.testing.assert_array_equal(s, z[f"sin_{D}_{P}"])


def test_attention_matches_reference_and_dense():
    n = 0
    for i, inp, want in F.attention_cases():
        assert inp["insha"].tobytes().hex() == sha(inp["q"]) + sha(inp["cache_k"]), "input drift"
        slots = A.table_slots(inp["block_ids"], inp["block_size"], inp["ctx"])
        got = A.paged_attention(inp["q"], inp["cache_k"], inp["cache_v"], slots, inp["n_kv"], inp["scale"])
        # the reference's own tolerance (tests/test_attention.py:57)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)
        dense = A.dense_attention(inp["q"], inp["cache_k"][slots], inp["cache_v"][slots], inp["n_kv"],
                                  inp["scale"])
        np.testing.assert_allclose(want, dense, rtol=1e-4, atol=1e-5)
        n += 1
    assert n == 27 + 12


def test_table_slots_follow_the_block_table():
    assert A.table_slots([3, 0], 4, 6).tolist() == [12, 13, 14, 15, 0, 1]
    assert A.table_slots([7], 16, 0).tolist() == []


@pytest.mark.parametrize("name,bs", [("replay_bench.npz", 16), ("replay_spec.npz", 4)])
def test_oracle_replays_reference_logits(name, bs):
    cfg = M.Shape(vocab_size=261, **F.BENCH)
    run = R.OracleRunner(cfg, M.seeded_weights(cfg), 512, bs)
    for seqs, cow, want in F.replay_steps(name):
        got, rows = run.execute(seqs, cow)
        assert got.shape == want.shape
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-5 * np.abs(want).max())


def test_sampling_fixtures():
    z = F.load("sampling.npz")
    rows, ps, keep = z["rows"], z["top_p"], z["keep"]
    for i in range(len(rows)):
        for j, p in enumerate(ps):
            np.testing.assert_array_equal(SP.top_p_keep(rows[i].copy(), float(p)), keep[i, j])
    seen_all = z["greedy_seen"]
    o = 0
    for (i, pen, mint, ngen, tok, nseen) in z["greedy"]:
        seen = seen_all[o:o + int(nseen)]
        o += int(nseen)
        got = SP.greedy(rows[int(i)], eos_id=257, num_generated=int(ngen), min_tokens=int(mint),
                        seen=seen, penalty=float(pen))
        assert got == int(tok)
    lo = to = do = 0
    for k, nt, acc in zip(z["verify_k"], z["verify_ntok"], z["verify_accepted"]):
        lg = z["verify_logits"][lo:lo + k + 1]
        dr = z["verify_drafts"][do:do + k].tolist()
        toks, a = SP.verify(lg, dr)
        assert a == acc and toks == z["verify_tokens"][to:to + nt].tolist()
        lo += k + 1
        do += k
        to += nt


def full_sampling_rows():
    """Yield (row index, logits, kwargs of oracle.sampling.sample_with_uniform,
    the reference's pick, keep set, probs) for every row of sampling_full.npz."""
    z = F.load("sampling_full.npz")
    o = 0
    eos = int(z["eos"])
    for i, (t, k, p, mint, ngen, pen, seed, nseen) in enumerate(z["params"]):
        seen = z["seen"][o:o + int(nseen)]
        o += int(nseen)
        kw = dict(temperature=float(t), top_k=int(k), top_p=float(p), u=float(z["u"][i]), eos_id=eos,
                  num_generated=int(ngen), min_tokens=int(mint), seen=seen, penalty=float(pen))
        yield i, z["rows"][i], kw, int(z["picks"][i]), z["keep"][i], z["probs"][i]


def test_full_sampler_matches_the_reference():
    """Temperature rows with EOS masks, repetition penalties, top-k and top-p:
    the oracle's sampler, given the uniform the reference's generator handed
    numpy's choice(), picks the reference's token and keeps its keep set."""
    n = masked = penalised = 0
    for i, row, kw, pick, keep, probs in full_sampling_rows():
        assert kw["u"] == np.random.default_rng(int(1000 + i)).random()
        tok, kept, pr = SP.sample_with_uniform(row, **kw)
        assert tok == pick, i
        np.testing.assert_array_equal(kept, keep)
        np.testing.assert_allclose(pr, probs, rtol=1e-6, atol=1e-9)
        assert keep[tok]
        masked += kw["num_generated"] < kw["min_tokens"]
        penalised += kw["penalty"] != 1.0 and len(kw["seen"]) > 0
        n += 1
    assert n == 96 and masked >= 10 and penalised >= 40
