"""CPU: the library's SIMT kernels, their own code, on the host.

csrc/sampling_kernels.cuh, norm_kernels.cuh, cache_kernels.cuh and
attention_kernels.cuh hold the device code of the sampling, row-wise,
KV-cache and generic attention kernels.
tests/kernels_host.cpp compiles it for the host, where each CTA runs as 256 cooperative fibers with CUDA's barrier and
warp-shuffle semantics (tests/simt_host.h). The kernels run with the grids
their launchers use, against the reference's fixtures. Every buffer sits
against a PROT_NONE guard page (tests/guarded.py), alternately after and
before it, so an out-of-bounds read or write stops the test; and every test
runs under two thread schedules (the default, and a seeded shuffle after
every barrier) to expose order-dependent reads:
  * greedy_kernel, on the reference's greedy cases (EOS mask under
    min_tokens, repetition penalty): its pick is the reference's, with
    aligned rows (vector path) and unaligned rows (scalar path); rows past the
    device row count are left untouched;
  * top_p_kernel, on the 96 rows of sampling_full.npz in one launch read
    through a shuffled row index: the reference's pick (except within 1e-5 of
    a CDF boundary) inside the reference's keep set; an index outside the
    logits yields -1. At the Llama-3 vocabulary with top-k and top-p it
    matches the oracle;
  * accept_kernel, on the reference's verify cases: the accepted counts;
  * rmsnorm_kernel against the oracle's rms_norm over gathered rows; the
    embedding (ids outside the vocabulary give zeros) and RoPE bit-identical
    to the oracle; the bf16 model's embedding and fused add + RMSNorm;
    argmax_rows with ties and padding;
  * reshape_and_cache (fp32 and bf16) and copy_blocks against the oracle's
    flat-slot cache, with slots and pairs outside the cache skipped;
  * the generic varlen attention kernel (and its split-K merge) against a
    float64 restatement of the reference's attention: C1 decode rows up to
    1300 keys, chunked-prefill tiles mixed with decode rows, the C3 shape
    (32 heads / 8 KV heads / D 128, 4096 keys), GQA 1 to 8, block sizes 1 to
    64, fp32 and bf16.
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
def _harness(tmp_path_factory):
    from tests.host_build import build_harness

    lib = build_harness("kernels_host", str(tmp_path_factory.mktemp("kernels")))
    if lib is None:
        pytest.skip("g++ is not available")
    lib.run_greedy.argtypes = [P, I, I, I, P, I, P, P, P, P]
    lib.run_top_p.argtypes = [P, I, I, I, I, P, P, I, P, P, P, P, P, P, P]
    lib.run_accept.argtypes = [P, P, P, I, P, P]
    lib.set_schedule_seed.argtypes = [ctypes.c_uint64]
    return lib


@pytest.fixture(scope="module", params=[0, 0x9E3779B97F4A7C15], ids=["schedule-default", "schedule-shuffled"])
def k(_harness, request):
    """Every kernel test runs twice: with the emulation's default schedule and
    with its seeded variation (a random thread continues after each barrier),
    so a read that races with another thread's write between two barriers
    meets two different orders."""
    _harness.set_schedule_seed(request.param)
    yield _harness
    _harness.set_schedule_seed(0)


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


# ---- row-wise kernels (csrc/norm_kernels.cuh) ---------------------------------------

def _bf16_bits(x):
    """float32 -> bf16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _bf16_float(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("dim", [64, 384])
def test_rmsnorm_kernel_against_the_oracle(k, dim):
    """fp32 RMSNorm (vllmlite/model.py:17-19) over gathered rows: within
    2 ulp-scale of the oracle (the sum of squares is reduced in another
    order), rows past the device row count untouched."""
    from oracle.model import rms_norm

    f = k.run_rmsnorm
    f.argtypes = [P, P, P, P, I, P, I, ctypes.c_float]
    rng = np.random.default_rng(dim)
    x = guarded(rng.standard_normal((50, dim)).astype(np.float32))
    w = guarded((1 + 0.1 * rng.standard_normal(dim)).astype(np.float32))
    idx = guarded(rng.permutation(50)[:40].astype(np.int32), "start")
    out = guarded(np.full((40, dim), -7, np.float32))
    rows = guarded(np.array([37], np.int32))
    assert f(ptr(x), ptr(idx), ptr(w), ptr(out), 40, ptr(rows), dim, 1e-5) == 0
    want = rms_norm(x[idx[:37]], w)
    np.testing.assert_allclose(out[:37], want, rtol=2e-6, atol=1e-7)
    assert (out[37:] == -7).all()


def test_embed_and_rope_kernels_against_the_oracle(k):
    """Embedding rows by token id (out-of-range ids give zeros), then RoPE on
    interleaved pairs (vllmlite/attention.py:28-37): bit-identical to the
    oracle, whose products and sums round the same way."""
    from oracle.attention import rope_tables, rotate

    emb_f = k.run_embed
    emb_f.argtypes = [P, P, P, I, P, I, I]
    rope_f = k.run_rope
    rope_f.argtypes = [P, P, P, P, I, I, I, I]
    rng = np.random.default_rng(3)
    V, H, D = 261, 8, 48
    dim = H * D
    emb = guarded(rng.standard_normal((V, dim)).astype(np.float32))
    tok = rng.integers(0, V, 30).astype(np.int32)
    tok[[4, 9]] = [-1, V]
    tok = guarded(tok, "start")
    x = guarded(np.full((30, dim), -7, np.float32))
    assert emb_f(ptr(emb), ptr(tok), ptr(x), 30, None, dim, V) == 0
    want = emb[np.clip(tok, 0, V - 1)]
    want[[4, 9]] = 0
    np.testing.assert_array_equal(x, want)
    cos, sin = rope_tables(D, 512)
    cos_g, sin_g = guarded(cos.astype(np.float32)), guarded(sin.astype(np.float32))
    pos = guarded(rng.integers(0, 512, 30).astype(np.int32), "start")
    before = x.copy().reshape(30, H, D)
    assert rope_f(ptr(x), ptr(pos), ptr(cos_g), ptr(sin_g), 30, H, D, 512) == 0
    np.testing.assert_array_equal(x.reshape(30, H, D), rotate(before, pos, cos, sin))


def test_bf16_embed_and_fused_add_rmsnorm(k):
    """The bf16 model's embedding (bf16 rows widened to fp32) and the fused
    x += add; out = bf16(x / rms * w) over gathered rows: x exact, out within
    one bf16 rounding of a float64 restatement."""
    emb_f = k.run_embed_bf16
    emb_f.argtypes = [P, P, P, I, P, I, I]
    f = k.run_rmsnorm_bf16
    f.argtypes = [P, P, P, P, P, I, P, I, ctypes.c_float]
    rng = np.random.default_rng(5)
    V, dim, T = 100, 256, 12
    table = _bf16_bits(rng.standard_normal((V, dim)))
    tok = guarded(rng.integers(0, V, T).astype(np.int32))
    x = guarded(np.full((T, dim), -7, np.float32))
    assert emb_f(ptr(guarded(table)), ptr(tok), ptr(x), T, None, dim, V) == 0
    np.testing.assert_array_equal(x, _bf16_float(table[tok]))
    add = _bf16_bits(rng.standard_normal((T, dim)))
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    idx = rng.permutation(T)[:8].astype(np.int32)
    x0 = x.copy()
    out = guarded(np.zeros((8, dim), np.uint16))
    assert f(ptr(x), ptr(guarded(add)), ptr(guarded(idx)), ptr(guarded(w)), ptr(out), 8, None, dim, 1e-5) == 0
    summed = x0 + _bf16_float(add)
    np.testing.assert_array_equal(x[idx], summed[idx])  # the gathered rows take the all-reduced partial
    xs = summed[idx].astype(np.float64)
    want = xs / np.sqrt((xs * xs).mean(1, keepdims=True) + 1e-5) * w
    np.testing.assert_allclose(_bf16_float(out), want, rtol=2 ** -8, atol=1e-6)


@pytest.mark.parametrize("ld", [264, 263])
def test_argmax_rows_kernel(k, ld):
    """(max, first index of the max) + offset per row, vector or scalar path."""
    f = k.run_argmax_rows
    f.argtypes = [P, I, P, I, I, I, P, P]
    rng = np.random.default_rng(ld)
    V, R = 261, 9
    x = rng.standard_normal((R, ld)).astype(np.float32)
    x[0, [5, 200]] = 9.0      # tie: the first index wins
    x[1, :] = 1.0             # all equal: index 0
    x[2, V:] = 100.0          # padding past the vocabulary is not read as a candidate
    val = guarded(np.zeros(R, np.float32))
    idx = guarded(np.zeros(R, np.int32))
    assert f(ptr(guarded(x)), R, None, V, ld, 1000, ptr(val), ptr(idx)) == 0
    np.testing.assert_array_equal(idx, x[:, :V].argmax(1) + 1000)
    np.testing.assert_array_equal(val, x[:, :V].max(1))


# ---- KV-cache kernels (csrc/cache_kernels.cuh) -------------------------------------

@pytest.mark.parametrize("f32", [1, 0])
def test_reshape_and_cache_and_copy_blocks(k, f32):
    """write_kv (vllmlite/attention.py:47-49) into the [block][kv head][offset][D]
    layout, skipping slots outside the cache, then copy-on-write block copies
    (vllmlite/runner.py:54-60) in every layer, skipping out-of-range pairs:
    the oracle's flat-slot cache, entry for entry."""
    from oracle.attention import scatter_kv
    from oracle.runner import copy_blocks

    w = k.run_reshape_and_cache
    w.argtypes = [P, P, P, P, P, I, I, I, I, I, I]
    c = k.run_copy_blocks
    c.argtypes = [P, P, P, I, I, I, I, I, I, I]
    rng = np.random.default_rng(f32)
    L, nb, n_kv, bs, D, T = 3, 10, 2, 4, 48 if f32 else 64, 13
    dt = np.float32 if f32 else np.uint16
    kv = [rng.standard_normal((T, n_kv, D)).astype(np.float32) for _ in range(2)]
    if not f32:
        kv = [_bf16_bits(a) for a in kv]
    slots = rng.choice(nb * bs, T, replace=False).astype(np.int32)
    slots[[2, 7]] = [-1, nb * bs]
    caches = [np.zeros((L, nb, n_kv, bs, D), dt) for _ in range(2)]
    gk, gv = guarded(caches[0]), guarded(caches[1], "start")
    layer = 1  # write into one layer's slice, as the forward does
    lk, lv = gk[layer], gv[layer]
    assert w(ptr(guarded(kv[0])), ptr(guarded(kv[1])), ptr(lk), ptr(lv), ptr(guarded(slots, "start")), T, n_kv, D,
             bs, nb, f32) == 0
    flat = [np.zeros((L, nb * bs, n_kv, D), dt) for _ in range(2)]
    ok = (slots >= 0) & (slots < nb * bs)
    scatter_kv(flat[0][layer], flat[1][layer], kv[0][ok], kv[1][ok], slots[ok])

    def as_flat(g):
        return g.transpose(0, 1, 3, 2, 4).reshape(L, nb * bs, n_kv, D)

    np.testing.assert_array_equal(as_flat(gk), flat[0])
    np.testing.assert_array_equal(as_flat(gv), flat[1])
    pairs = np.array([[slots[0] // bs, 9], [3, 0], [-1, 2], [4, nb]], np.int32)
    assert c(ptr(gk), ptr(gv), ptr(guarded(pairs)), len(pairs), L, nb, n_kv, bs, D, f32) == 0
    copy_blocks(flat[0], flat[1], [tuple(p) for p in pairs[:2]], bs)
    np.testing.assert_array_equal(as_flat(gk), flat[0])
    np.testing.assert_array_equal(as_flat(gv), flat[1])


# ---- generic paged attention (csrc/attention_kernels.cuh) --------------------------

def _attention_case(rng, qlens, ctxs, H, n_kv, D, bs, f32, spare=7):
    """Random q / K / V per sequence, K and V scattered into the
    [block][kv head][offset][D] cache through shuffled block tables."""
    S = len(qlens)
    W = max(-(-c // bs) for c in ctxs)
    nb = sum(-(-c // bs) for c in ctxs) + spare
    perm = rng.permutation(nb)
    tables = np.full((S, W), -1, np.int32)
    o = 0
    kc = np.zeros((nb, n_kv, bs, D), np.float32)
    vc = np.zeros_like(kc)
    dense = []
    for s, c in enumerate(ctxs):
        n = -(-c // bs)
        tables[s, :n] = perm[o:o + n]
        o += n
        k = rng.standard_normal((c, n_kv, D)).astype(np.float32)
        v = rng.standard_normal((c, n_kv, D)).astype(np.float32)
        if not f32:
            k, v = _bf16_float(_bf16_bits(k)), _bf16_float(_bf16_bits(v))
        for p in range(c):
            kc[tables[s, p // bs], :, p % bs] = k[p]
            vc[tables[s, p // bs], :, p % bs] = v[p]
        dense.append((k, v))
    T = sum(qlens)
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    if not f32:
        q = _bf16_float(_bf16_bits(q))
    cu = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    return q, kc, vc, tables, cu, np.asarray(ctxs, np.int32), dense, nb, W


@pytest.mark.parametrize("f32", [1, 0])
@pytest.mark.parametrize("H,n_kv,D,bs,qlens,ctxs,single", [
    (8, 4, 48, 16, [1] * 6, [1, 15, 16, 17, 300, 1300], 1),     # C1 decode rows, split-K past 512 keys
    (8, 4, 48, 16, [40, 1, 7, 16], [40, 200, 7, 33], 0),       # chunked prefill tiles mixed with decode rows
    (32, 8, 128, 16, [1] * 3, [4096, 517, 1], 1),              # C3 shape, 8 splits
    (6, 1, 64, 4, [9, 3], [30, 3], 0),                         # GQA 6, block 4
    (4, 4, 8, 1, [3, 1], [3, 9], 0),                           # MHA, block 1, head_dim 8
    (16, 2, 32, 64, [5, 1], [70, 64], 0),                      # n_rep 8, block 64
])
def test_generic_attention_kernel_against_float64(k, f32, H, n_kv, D, bs, qlens, ctxs, single):
    """The generic varlen kernel (vllmlite/attention.py:59-98 for a ragged
    batch: causal, GQA, online softmax, split-K with the merge kernel) against
    a float64 restatement of the reference's attention. Tolerance: fp32 paths
    2e-5 of the output scale, bf16 outputs one bf16 rounding (2^-8)."""
    from oracle.attention import dense_attention

    f = k.run_attention
    f.argtypes = [I, P, P, P, P, P, I, P, P, I, I, I, I, I, I, I, I, I, ctypes.c_float, P, ctypes.c_int64]
    rng = np.random.default_rng(D * 7 + len(qlens) + f32)
    q, kc, vc, tables, cu, ctx, dense, nb, W = _attention_case(rng, qlens, ctxs, H, n_kv, D, bs, f32)
    scale = 1.0 / np.sqrt(D)
    S, T = len(qlens), int(cu[-1])
    if f32:
        bufs = [guarded(a) for a in (q, kc, vc)]
        out = guarded(np.full((T, H, D), np.nan, np.float32))
    else:
        bufs = [guarded(_bf16_bits(a)) for a in (q, kc, vc)]
        out = guarded(np.zeros((T, H, D), np.uint16))
    splits = -(-max(ctxs) // 512)
    ws = guarded(np.zeros(splits * S * H * (D + 2), np.float32), "start")
    assert f(f32, ptr(bufs[0]), ptr(bufs[1]), ptr(bufs[2]), ptr(out), ptr(guarded(tables, "start")), W,
             ptr(guarded(cu)), ptr(guarded(ctx, "start")), S, max(qlens), single, max(ctxs), H, n_kv, D, bs, nb,
             scale, ptr(ws), ws.nbytes) == 0
    got = out if f32 else _bf16_float(out)
    for s in range(S):
        kk, vv = dense[s]
        want = dense_attention(q[cu[s]:cu[s + 1]], kk, vv, n_kv, scale)
        tol = 2e-5 if f32 else 2.0 ** -8
        np.testing.assert_allclose(got[cu[s]:cu[s + 1]], want, rtol=tol, atol=tol)


# ---- fp32 SIMT GEMM and its epilogues (csrc/gemm_f32_kernels.cuh) -----------------

GEMM_ARGS = [P, I, P, I, I, P, I, I, P, P, ctypes.c_int64, I]


def _gemm(k, name, extra):
    f = getattr(k, name)
    f.argtypes = GEMM_ARGS + extra
    return f


def _scratch(N):
    """The forward's split-K scratch for N columns (gemm_scratch_floats / counters)."""
    floats = -(-N // 64) * 64 * 64 * 8
    return guarded(np.zeros(floats, np.float32)), guarded(np.zeros(-(-N // 64) * 4, np.int32), "start")


def _gemm_tol(A, B):
    """fp32 accumulation bound against float64: K * eps * |A| |B|."""
    return A.shape[1] * 2.0 ** -23 * (np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64))


@pytest.mark.parametrize("M", [1, 5, 16, 17, 40, 64, 65, 130])
@pytest.mark.parametrize("split", [True, False])
def test_sgemm_store_and_residual(k, M, split):
    """C = A @ B (lm_head rows, columns past n_valid untouched) and C += A @ B
    (o_proj / down_proj residual) against float64, with the split-K path for
    small M when scratch is given (its counters end at zero for the next
    launch or graph replay), and rows past the device row count untouched."""
    store = _gemm(k, "run_sgemm_store", [P, I, I])
    resid = _gemm(k, "run_sgemm_residual", [P, I])
    rng = np.random.default_rng(M + 100 * split)
    K, N = 384, 264
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    Mv = max(1, M - 2)  # rows on the device counter
    part, cnt = _scratch(N) if split else (None, None)
    args = lambda: [ptr(guarded(A)), K, ptr(guarded(B, "start")), N, M, ptr(guarded(np.array([Mv], np.int32))), N, K,
                    ptr(part), ptr(cnt), part.size if split else 0, cnt.size if split else 0]
    C = guarded(np.full((M, N), 7.0, np.float32))
    assert store(*args(), ptr(C), N, 261) == 0
    want = A.astype(np.float64) @ B.astype(np.float64)
    tol = _gemm_tol(A, B)
    assert (np.abs(C[:Mv, :261] - want[:Mv, :261]) <= tol[:Mv, :261] + 1e-7).all()
    assert (C[:Mv, 261:] == 7.0).all() and (C[Mv:] == 7.0).all()
    R = guarded(np.ones((M, N), np.float32))
    assert resid(*args(), ptr(R), N) == 0
    assert (np.abs(R[:Mv] - (1.0 + want[:Mv])) <= tol[:Mv] + 1e-6).all() and (R[Mv:] == 1.0).all()
    if split:
        assert (cnt == 0).all()


@pytest.mark.parametrize("M", [3, 33, 100])
def test_sgemm_swiglu(k, M):
    """Gate/up columns interleaved (gate_j, up_j): out_j = silu(gate_j) * up_j
    (vllmlite/model.py:22-23, :117)."""
    from oracle.model import silu

    f = _gemm(k, "run_sgemm_swiglu", [P, I])
    rng = np.random.default_rng(M)
    K, F = 384, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((K, 2 * F)) / np.sqrt(K)).astype(np.float32)
    part, cnt = _scratch(2 * F)
    out = guarded(np.zeros((M, F), np.float32))
    assert f(ptr(guarded(A)), K, ptr(guarded(B)), 2 * F, M, None, 2 * F, K, ptr(part), ptr(cnt), part.size, cnt.size,
             ptr(out), F) == 0
    y = A.astype(np.float64) @ B.astype(np.float64)
    want = silu(y[:, 0::2]) * y[:, 1::2]
    np.testing.assert_allclose(out, want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("H,n_kv,D,bs", [(8, 4, 48, 16), (4, 2, 64, 4), (32, 8, 128, 16)])
def test_sgemm_qkv_epilogue(k, H, n_kv, D, bs):
    """The QKV projection's epilogue: RoPE on the q and k columns at each
    token's position (interleaved pairs, vllmlite/attention.py:28-37), q to its
    buffer, k and v into the paged cache at the token's slot (write_kv,
    attention.py:47-49); tokens with slot -1 write no K/V."""
    from oracle.attention import rope_tables, rotate

    f = _gemm(k, "run_sgemm_qkv", [P, P, P, P, P, P, P, I, I, I, I, I, ctypes.c_int64])
    rng = np.random.default_rng(D)
    T, d, nb, max_pos = 21, 128, 12, 256
    N = (H + 2 * n_kv) * D
    A = rng.standard_normal((T, d)).astype(np.float32)
    B = (rng.standard_normal((d, N)) / np.sqrt(d)).astype(np.float32)
    pos = rng.integers(0, max_pos, T).astype(np.int32)
    slot = rng.choice(nb * bs, T, replace=False).astype(np.int32)
    slot[3] = -1
    cos, sin = rope_tables(D, max_pos)
    part, cnt = _scratch(N)
    q_out = guarded(np.zeros((T, H * D), np.float32))
    kc = guarded(np.zeros((nb, n_kv, bs, D), np.float32))
    vc = guarded(np.zeros((nb, n_kv, bs, D), np.float32), "start")
    assert f(ptr(guarded(A)), d, ptr(guarded(B)), N, T, None, N, d, ptr(part), ptr(cnt), part.size, cnt.size,
             ptr(q_out), ptr(kc), ptr(vc), ptr(guarded(pos)), ptr(guarded(slot)), ptr(guarded(cos.astype(np.float32))),
             ptr(guarded(sin.astype(np.float32))), H, n_kv, D, bs, max_pos, nb * bs) == 0
    y = (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)
    q = rotate(y[:, :H * D].reshape(T, H, D), pos, cos, sin)
    kk = rotate(y[:, H * D:(H + n_kv) * D].reshape(T, n_kv, D), pos, cos, sin)
    vv = y[:, (H + n_kv) * D:].reshape(T, n_kv, D)
    np.testing.assert_allclose(q_out.reshape(T, H, D), q, rtol=1e-4, atol=1e-5)
    for t in range(T):
        if slot[t] < 0:
            continue
        b, o = divmod(int(slot[t]), bs)
        np.testing.assert_allclose(kc[b, :, o], kk[t], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(vc[b, :, o], vv[t], rtol=1e-4, atol=1e-5)
    written = {divmod(int(s), bs) for s in slot if s >= 0}
    for b in range(nb):
        for o in range(bs):
            if (b, o) not in written:
                assert not kc[b, :, o].any() and not vc[b, :, o].any()
