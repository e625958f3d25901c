"""CPU: the library's sampling kernels, their own code, on the host.

csrc/sampling_kernels.cuh holds the device code of greedy_kernel,
top_p_kernel and accept_kernel. tests/kernels_host.cpp compiles it for the
host, where each CTA runs as 256 cooperative fibers with CUDA's barrier and
warp-shuffle semantics (tests/simt_host.h). The kernels run with the grids
their launchers use, against the reference's fixtures. Every buffer sits
against a PROT_NONE guard page (tests/guarded.py), alternately after and
before it, so an out-of-bounds read or write stops the test:
  * greedy_kernel, on the reference's greedy cases (EOS mask under
    min_tokens, repetition penalty): its pick is the reference's, with
    aligned rows (vector path) and unaligned rows (scalar path); rows past the
    device row count are left untouched;
  * top_p_kernel, on the 96 rows of sampling_full.npz in one launch read
    through a shuffled row index: the reference's pick (except within 1e-5 of
    a CDF boundary) inside the reference's keep set; an index outside the
    logits yields -1. At the Llama-3 vocabulary with top-k and top-p it
    matches the oracle;
  * accept_kernel, on the reference's verify cases: the accepted counts.
"""

import ctypes

import numpy as np
import pytest

from oracle import sampling as SP
from tests import fixtures as F
from tests.guarded import guarded, ptr
from tests.test_oracle_golden import full_sampling_rows

P = ctypes.c_void_p
I = ctypes.c_int


@pytest.fixture(scope="module")
def k(tmp_path_factory):
    from tests.host_build import build_harness

    lib = build_harness("kernels_host", str(tmp_path_factory.mktemp("kernels")))
    if lib is None:
        pytest.skip("g++ is not available")
    lib.run_greedy.argtypes = [P, I, I, I, P, I, P, P, P, P]
    lib.run_top_p.argtypes = [P, I, I, I, I, P, P, I, P, P, P, P, P, P, P]
    lib.run_accept.argtypes = [P, P, P, I, P, P]
    return lib


def bitmaps(seen_lists, vocab):
    words = (vocab + 31) // 32
    b = np.zeros((len(seen_lists), words), np.uint32)
    for j, seen in enumerate(seen_lists):
        for t in set(int(x) for x in seen):
            b[j, t >> 5] |= np.uint32(1 << (t & 31))
    return b


@pytest.mark.parametrize("ld,side", [(264, "end"), (261, "start")])
def test_greedy_kernel_on_reference_cases(k, ld, side):
    z = F.load("sampling.npz")
    rows, V = z["rows"], z["rows"].shape[1]
    cases, seen_all = z["greedy"], z["greedy_seen"]
    n = len(cases)
    logits = np.zeros((n, ld), np.float32)
    mask = np.zeros(n, np.uint8)
    pen = np.ones(n, np.float32)
    seen, want, o = [], [], 0
    for j, (i, p, mint, ngen, tok, nseen) in enumerate(cases):
        logits[j, :V] = rows[int(i)]
        mask[j] = ngen < mint
        pen[j] = p
        seen.append(seen_all[o:o + int(nseen)])
        o += int(nseen)
        want.append(int(tok))
    bits = bitmaps(seen, V)
    out = guarded(np.full(n + 3, -7, np.int32), side)
    count = guarded(np.array([n], np.int32), side)
    args = [guarded(a, side) for a in (logits, mask, pen, bits)]
    assert k.run_greedy(ptr(args[0]), n + 3, V, ld, ptr(args[1]), 257, ptr(args[2]), ptr(args[3]), ptr(count),
                        ptr(out)) == 0
    assert out[:n].tolist() == want
    assert out[n:].tolist() == [-7] * 3  # rows past the device row count are not written
    assert mask.any() and (pen != 1).any()


def test_top_p_kernel_on_the_reference_sampler_fixture(k):
    data = list(full_sampling_rows())
    n, V = len(data), data[0][1].size
    ld = 264
    logits = np.zeros((n, ld), np.float32)
    order = np.random.default_rng(1).permutation(n)  # call row j reads logits row order[j]
    for i, row, kw, pick, keep, probs in data:
        logits[i, :V] = row
    R = n + 1  # one more call row, reading outside the logits
    row_index = np.append(order, n).astype(np.int32)
    temp = np.ones(R, np.float32)
    top_k = np.zeros(R, np.int32)
    top_p = np.ones(R, np.float32)
    u = np.zeros(R, np.float64)
    mask = np.zeros(R, np.uint8)
    pen = np.ones(R, np.float32)
    seen = [[] for _ in range(R)]
    for j, i in enumerate(order):
        _, _, kw, _, _, _ = data[i]
        temp[j], top_k[j], top_p[j], u[j] = kw["temperature"], kw["top_k"], kw["top_p"], kw["u"]
        mask[j] = kw["num_generated"] < kw["min_tokens"]
        pen[j] = kw["penalty"]
        seen[j] = kw["seen"]
    bits = bitmaps(seen, V)
    out = guarded(np.full(R, -7, np.int32))
    g = [guarded(a, "start") for a in (logits, row_index, mask, pen, bits, temp, top_k, top_p, u)]
    assert k.run_top_p(ptr(g[0]), R, V, ld, n, ptr(g[1]), ptr(g[2]), data[0][2]["eos_id"], ptr(g[3]), ptr(g[4]),
                       ptr(g[5]), ptr(g[6]), ptr(g[7]), ptr(g[8]), ptr(out)) == 0
    assert out[n] == -1
    exact = 0
    for j, i in enumerate(order):
        _, _, kw, pick, keep, probs = data[i]
        tok = int(out[j])
        assert 0 <= tok < V and keep[tok], (i, tok)
        cdf = np.cumsum(probs.astype(np.float64))
        cdf /= cdf[-1]
        if np.abs(cdf - kw["u"]).min() > 1e-5:
            assert tok == pick, (i, tok, pick)
            exact += 1
    assert exact >= n - 2


@pytest.mark.parametrize("top_k,top_p", [(50, 1.0), (0, 0.9), (128255, 0.8)])
def test_top_p_kernel_llama3_vocabulary(k, top_k, top_p):
    V = ld = 128256
    rng = np.random.default_rng(top_k)
    x = guarded((rng.standard_normal((2, V)) * 3).astype(np.float32))
    us = np.array([0.37, 0.999], np.float64)
    out = guarded(np.full(2, -7, np.int32))
    g = [guarded(a) for a in (np.full(2, 0.8, np.float32), np.full(2, top_k, np.int32),
                              np.full(2, top_p, np.float32), us)]
    assert k.run_top_p(ptr(x), 2, V, ld, 2, None, None, -1, None, None, ptr(g[0]), ptr(g[1]), ptr(g[2]), ptr(g[3]),
                       ptr(out)) == 0
    for r in range(2):
        want, _, _ = SP.sample_with_uniform(x[r], 0.8, top_k, top_p, float(us[r]))
        assert out[r] == want


def test_accept_kernel_on_reference_verify_cases(k):
    z = F.load("sampling.npz")
    ks, lg = z["verify_k"], z["verify_logits"]
    picks = lg.argmax(1).astype(np.int32)  # the greedy row picks the accept rule reads
    cu = np.concatenate([[0], np.cumsum(ks + 1)]).astype(np.int32)
    doff = np.concatenate([[0], np.cumsum(ks)[:-1]]).astype(np.int32)
    S = len(ks)
    acc = guarded(np.full(S, -7, np.int32))
    g = [guarded(a) for a in (cu, z["verify_drafts"].astype(np.int32), doff, picks)]
    assert k.run_accept(ptr(g[0]), ptr(g[1]), ptr(g[2]), S, ptr(g[3]), ptr(acc)) == 0
    assert acc.tolist() == z["verify_accepted"].tolist()
