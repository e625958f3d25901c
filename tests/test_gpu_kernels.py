"""GPU: every kernel through the C ABI against the oracle / golden vectors.

Tolerances: fp32 kernels use the reference's own attention tolerance
(rtol 1e-4, atol 1e-5, tests/test_attention.py:57 of the reference) or tighter;
bf16 attention (fp32 accumulate, bf16 output) is checked against a float64
oracle on the same bf16 inputs within rtol 2e-2, atol 2e-2. Integer and index
work (slots, block copies, token picks) must be bit-exact.
"""

import numpy as np
import pytest

from oracle import attention as A
from oracle import model as OM
from oracle import runner as OR
from oracle import sampling as SP
from tests import fixtures as F

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    return torch.device("cuda", 0)


def to_lib_layout(cache, bs):
    """Reference cache [slots, n_kv, D] -> library [NB, n_kv, bs, D]."""
    slots, n_kv, D = cache.shape
    return np.ascontiguousarray(cache.reshape(slots // bs, bs, n_kv, D).transpose(0, 2, 1, 3))


def test_attention_golden_cases_dropin(dev):
    """The NumPy drop-in paged_attention on every reference test case."""
    from vllt.ops import paged_attention

    for i, inp, want in F.attention_cases():
        slots = A.table_slots(inp["block_ids"], inp["block_size"], inp["ctx"])
        got = paged_attention(inp["q"], inp["cache_k"], inp["cache_v"], slots, inp["n_kv"], inp["scale"])
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5, err_msg=f"case {i}")


def test_attention_golden_cases_paged_layout(dev):
    """Same cases through block tables in the library's paged layout."""
    from vllt.ops import paged_attention_varlen

    for i, inp, want in F.attention_cases():
        bs = inp["block_size"]
        ck = torch.from_numpy(to_lib_layout(inp["cache_k"], bs)).to(dev)
        cv = torch.from_numpy(to_lib_layout(inp["cache_v"], bs)).to(dev)
        q = torch.from_numpy(inp["q"]).to(dev)
        got = paged_attention_varlen(q, ck, cv, np.asarray([inp["block_ids"]]), [0, q.shape[0]],
                                     [inp["ctx"]], inp["scale"]).cpu().numpy()
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5, err_msg=f"case {i}")


def ragged_batch(rng, H, KV, D, bs, qlens, ctxs, dtype=np.float32):
    nb_need = [(c + bs - 1) // bs for c in ctxs]
    total = sum(nb_need) + 7
    perm = rng.permutation(total)
    tables, o = [], 0
    for n in nb_need:
        tables.append(perm[o:o + n].tolist())
        o += n
    W = max(nb_need)
    tab = np.zeros((len(ctxs), W), np.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = t
    ck = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
    cv = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
    q = rng.standard_normal((sum(qlens), H, D)).astype(np.float32)
    if dtype != np.float32:  # round inputs to bf16 so both sides see the same values
        r = lambda a: torch.from_numpy(a).bfloat16().float().numpy()
        ck, cv, q = r(ck), r(cv), r(q)
    return q, ck, cv, tables, tab


@pytest.mark.parametrize("H,KV,D,bs,dtype", [
    (8, 4, 48, 16, "f32"), (4, 2, 16, 4, "f32"), (6, 1, 8, 1, "f32"), (8, 8, 64, 16, "f32"),
    (32, 8, 128, 16, "f32"), (32, 8, 128, 16, "bf16"), (8, 4, 48, 16, "bf16")])
def test_attention_varlen_mixed_batch(dev, H, KV, D, bs, dtype):
    """Decode, chunked-prefill and verify rows in one launch, including a
    context long enough to take the split-K path."""
    from vllt.ops import paged_attention_varlen

    rng = np.random.default_rng(H * 100 + D + bs)
    qlens = [1, 1, 7, 1, 33, 5, 1, 64, 2]
    ctxs = [1, 300, 40, 1500, 33, 700, 17, 1100, 16]
    npdt = np.float32 if dtype == "f32" else "bf16"
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, bs, qlens, ctxs, npdt)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    tq = torch.from_numpy(q).to(dev, tdt)
    tk = torch.from_numpy(to_lib_layout(ck, bs)).to(dev, tdt)
    tv = torch.from_numpy(to_lib_layout(cv, bs)).to(dev, tdt)
    cu = np.concatenate([[0], np.cumsum(qlens)])
    scale = 1.0 / np.sqrt(D)
    got = paged_attention_varlen(tq, tk, tv, tab, cu, ctxs, scale).float().cpu().numpy()
    for i, (ql, c) in enumerate(zip(qlens, ctxs)):
        slots = A.table_slots(tables[i], bs, c)
        if dtype == "f32":
            want = A.paged_attention(q[cu[i]:cu[i + 1]], ck, cv, slots, KV, scale)
            np.testing.assert_allclose(got[cu[i]:cu[i + 1]], want, rtol=1e-4, atol=1e-5, err_msg=f"seq {i}")
        else:
            want = A.dense_attention(q[cu[i]:cu[i + 1]], ck[slots], cv[slots], KV, scale)
            np.testing.assert_allclose(got[cu[i]:cu[i + 1]], want, rtol=2e-2, atol=2e-2, err_msg=f"seq {i}")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_reshape_and_cache_is_exact(dev, dtype):
    from vllt.ops import write_kv

    rng = np.random.default_rng(1)
    nb, KV, bs, D, T = 40, 4, 16, 48, 77
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    ref_k = rng.standard_normal((nb * bs, KV, D)).astype(np.float32)
    ref_v = rng.standard_normal((nb * bs, KV, D)).astype(np.float32)
    ref_k = torch.from_numpy(ref_k).to(tdt).float().numpy()
    ref_v = torch.from_numpy(ref_v).to(tdt).float().numpy()
    k = torch.from_numpy(rng.standard_normal((T, KV, D)).astype(np.float32)).to(tdt)
    v = torch.from_numpy(rng.standard_normal((T, KV, D)).astype(np.float32)).to(tdt)
    slots = rng.permutation(nb * bs)[:T]
    slots[5] = -1  # skipped
    ck = torch.from_numpy(to_lib_layout(ref_k, bs)).to(dev, tdt)
    cv = torch.from_numpy(to_lib_layout(ref_v, bs)).to(dev, tdt)
    write_kv(ck, cv, k.to(dev), v.to(dev), slots)
    keep = slots >= 0
    A.scatter_kv(ref_k, ref_v, k.float().numpy()[keep], v.float().numpy()[keep], slots[keep])
    np.testing.assert_array_equal(ck.float().cpu().numpy(), to_lib_layout(ref_k, bs))
    np.testing.assert_array_equal(cv.float().cpu().numpy(), to_lib_layout(ref_v, bs))


def test_copy_blocks_is_exact(dev):
    from vllt.ops import copy_blocks

    rng = np.random.default_rng(2)
    L, nb, KV, bs, D = 3, 20, 4, 16, 48
    rk = rng.standard_normal((L, nb * bs, KV, D)).astype(np.float32)
    rv = rng.standard_normal((L, nb * bs, KV, D)).astype(np.float32)
    tk = torch.from_numpy(np.stack([to_lib_layout(rk[l], bs) for l in range(L)])).to(dev)
    tv = torch.from_numpy(np.stack([to_lib_layout(rv[l], bs) for l in range(L)])).to(dev)
    pairs = [(3, 7), (0, 19), (12, 4)]
    copy_blocks(tk, tv, pairs)
    OR.copy_blocks(rk, rv, pairs, bs)
    np.testing.assert_array_equal(tk.cpu().numpy(), np.stack([to_lib_layout(rk[l], bs) for l in range(L)]))
    np.testing.assert_array_equal(tv.cpu().numpy(), np.stack([to_lib_layout(rv[l], bs) for l in range(L)]))


def test_rmsnorm_rope_sgemm(dev):
    from vllt.ops import apply_rope, matmul, rms_norm
    from vllt.model import rope_tables

    rng = np.random.default_rng(3)
    x = rng.standard_normal((37, 384)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(384)).astype(np.float32)
    got = rms_norm(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)).cpu().numpy()
    np.testing.assert_allclose(got, OM.rms_norm(x, w), rtol=2e-6, atol=1e-6)
    idx = np.asarray([5, 0, 36, 5], np.int32)
    got = rms_norm(torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), idx=idx).cpu().numpy()
    np.testing.assert_allclose(got, OM.rms_norm(x[idx], w), rtol=2e-6, atol=1e-6)

    cos, sin = rope_tables(48, 512)
    xr = rng.standard_normal((29, 8, 48)).astype(np.float32)
    pos = rng.integers(0, 512, size=29)
    t = torch.from_numpy(xr.copy()).to(dev)
    apply_rope(t, pos, torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev))
    np.testing.assert_array_equal(t.cpu().numpy(), A.rotate(xr, pos, cos, sin))

    for M, N, K in ((1, 768, 384), (16, 2048, 384), (100, 384, 1024), (1024, 264, 384), (300, 64, 64)):
        a = rng.standard_normal((M, K)).astype(np.float32)
        b = rng.standard_normal((K, N)).astype(np.float32)
        got = matmul(torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)).cpu().numpy()
        want = a.astype(np.float64) @ b.astype(np.float64)
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-4 * np.sqrt(K) * 1e-1)


def test_sampling_kernels_match_reference(dev):
    from vllt.ops import greedy, sample_top_p, verify

    z = F.load("sampling.npz")
    rows = z["rows"]
    R, V = rows.shape
    # greedy with min_tokens EOS mask and repetition penalty (sampling.py:41-57)
    mask = np.zeros(R, np.uint8)
    pen = np.ones(R, np.float32)
    bits = np.zeros((R, (V + 31) // 32), np.uint32)
    o = 0
    for (i, p, mint, ngen, tok, nseen) in z["greedy"]:
        i = int(i)
        mask[i] = 1 if ngen < mint else 0
        pen[i] = p
        for t in np.unique(z["greedy_seen"][o:o + int(nseen)]):
            bits[i, t >> 5] |= np.uint32(1) << np.uint32(t & 31)
        o += int(nseen)
    got = greedy(torch.from_numpy(rows).to(dev), eos_mask=torch.from_numpy(mask).to(dev),
                 penalty=torch.from_numpy(pen).to(dev), seen_bits=torch.from_numpy(bits).to(dev)).cpu().numpy()
    assert got.tolist() == [int(t) for t in z["greedy"][:, 4]]
    # batched verify (speculative.py:86-100)
    k, nt, acc = z["verify_k"], z["verify_ntok"], z["verify_accepted"]
    cu = np.concatenate([[0], np.cumsum(k + 1)])
    doff = np.concatenate([[0], np.cumsum(k)[:-1]])
    toks, a = verify(torch.from_numpy(z["verify_logits"]).to(dev), cu, z["verify_drafts"], doff)
    toks, a = toks.cpu().numpy(), a.cpu().numpy()
    assert a.tolist() == acc.tolist()
    to = 0
    for s in range(len(k)):
        assert toks[cu[s]:cu[s] + nt[s]].tolist() == z["verify_tokens"][to:to + nt[s]].tolist()
        to += nt[s]
    # top-p: the drawn token always lies in the reference's keep set, and a
    # draw with the same uniform lands on numpy's choice() pick
    ps = z["top_p"]
    for j, p in enumerate(ps):
        u = np.random.default_rng(j).random(R).astype(np.float32)
        out = sample_top_p(torch.from_numpy(rows).to(dev), torch.ones(R, device=dev),
                           torch.zeros(R, dtype=torch.int32, device=dev), torch.full((R,), float(p), device=dev),
                           torch.from_numpy(u).to(dev)).cpu().numpy()
        for i in range(R):
            keep = z["keep"][i, j]
            assert keep[out[i]], (i, p)
            lg = np.where(keep, rows[i], -np.inf)
            pr = np.exp(lg - lg.max())
            pr /= pr.sum()
            cdf = np.cumsum(pr.astype(np.float64))
            cdf /= cdf[-1]
            want = int(np.searchsorted(cdf, float(u[i]), side="right"))
            if abs(cdf[min(want, V - 1)] - u[i]) > 1e-5 and (want == 0 or abs(cdf[want - 1] - u[i]) > 1e-5):
                assert out[i] == want, (i, p)


def test_full_sampler_matches_reference(dev):
    """vllt_sample_top_p on temperature rows with min_tokens EOS masks,
    repetition penalties, top-k and top-p (sampling_full.npz, written by the
    reference's sample()): given the uniform the reference's generator handed
    numpy's choice(), every device pick lies in the reference's keep set and
    equals the reference's pick unless u lies within 1e-5 of a CDF boundary
    (the device sums the float32 probabilities in another order). Rows are
    read through a shuffled row index; an index outside the buffer gives -1."""
    from tests.test_oracle_golden import full_sampling_rows
    from vllt.engine import seen_bitmaps
    from vllt.ops import sample_top_p

    items = list(full_sampling_rows())
    n = len(items)
    V = items[0][1].size
    perm = np.random.default_rng(4).permutation(n)
    logits = np.stack([items[j][1] for j in perm])  # row r of the buffer holds fixture row perm[r]
    where = np.argsort(perm)  # fixture row i sits at buffer row where[i]
    kw = [it[2] for it in items]
    f32 = lambda a: torch.tensor(np.asarray(a, np.float32), device=dev)
    temp = f32([k["temperature"] for k in kw])
    top_k = torch.tensor([k["top_k"] for k in kw], dtype=torch.int32, device=dev)
    top_p = f32([k["top_p"] for k in kw])
    u = torch.tensor([k["u"] for k in kw], dtype=torch.float64, device=dev)
    mask = torch.tensor([k["num_generated"] < k["min_tokens"] for k in kw], dtype=torch.uint8, device=dev)
    pen = f32([k["penalty"] for k in kw])
    seqs = [type("S", (), {"token_ids": list(k["seen"])})() for k in kw]
    bits = torch.from_numpy(seen_bitmaps(seqs, V)).to(dev)
    out = sample_top_p(torch.from_numpy(logits).to(dev), temp, top_k, top_p, u, row_index=where,
                       eos_mask=mask, eos_id=kw[0]["eos_id"], penalty=pen, seen_bits=bits).cpu().numpy()
    exact = 0
    for i, row, k, pick, keep, probs in items:
        assert keep[out[i]], (i, out[i])
        cdf = np.cumsum(probs.astype(np.float64))
        cdf /= cdf[-1]
        if np.abs(cdf - k["u"]).min() > 1e-5:
            assert out[i] == pick, (i, out[i], pick)
            exact += 1
    assert exact >= n - 2
    bad = sample_top_p(torch.from_numpy(logits).to(dev), temp[:2], top_k[:2], top_p[:2], u[:2],
                       row_index=np.asarray([0, n], np.int32)).cpu().numpy()
    assert bad[1] == -1 and bad[0] >= 0


def test_batch_meta_matches_reference_flatten(dev):
    """Device-built positions / slots / logit rows equal runner.py:66-90."""
    import ctypes

    from vllt import _lib
    from vllt.runner import pack_step, tile_positions

    L = _lib.lib()
    for seqs, cow, _ in F.replay_steps("replay_spec.npz"):
        bs = 4
        out = F.as_scheduler_output(seqs, cow)
        rec, bounds, rows, (S, T, R, W) = pack_step(out, bs, 512, 261, 512, tile_positions(2))
        caps = _lib.Caps(S + 3, T + 5, R + 2, W + 1)
        meta = torch.zeros(L.vllt_meta_bytes(ctypes.byref(caps)) // 4, dtype=torch.int32, device=dev)
        drec = torch.from_numpy(rec).to(dev)
        _lib.check(L.vllt_build_batch_meta(drec.data_ptr(), ctypes.byref(caps), bs, 512, 2, meta.data_ptr(),
                                           _lib.stream_handle()))
        torch.cuda.synchronize()
        base = meta.data_ptr()

        def field(i, n):
            off = (L.vllt_meta_field(ctypes.c_void_p(base), ctypes.byref(caps), i) - base) // 4
            return meta[off:off + n].cpu().numpy()

        cnt = field(0, 16)
        assert cnt[:4].tolist() == [S, T, R, W] and cnt[7] == 0
        tok, pos, smeta, last, orows = OR.flatten(seqs, bs)
        assert field(4, T).tolist() == pos.tolist()
        wslots = np.concatenate([m[2] for m in smeta])
        assert field(5, T).tolist() == wslots.tolist()
        assert field(6, R).tolist() == last.tolist()
        assert field(1, S + 1).tolist() == [0] + np.cumsum([s["n"] for s in seqs]).tolist()
        assert cnt[4] == bounds.decode_seqs and cnt[5] == bounds.tiles


def test_batch_meta_flags_bad_tables_without_faulting(dev):
    import ctypes

    from vllt import _lib

    L = _lib.lib()
    caps = _lib.Caps(4, 16, 16, 4)
    rec = np.asarray([1, 3, 1, 1, 0, 3, 1, 256, 1, 2, 777], np.int32)  # block 777 >= num_blocks
    meta = torch.zeros(L.vllt_meta_bytes(ctypes.byref(caps)) // 4, dtype=torch.int32, device=dev)
    drec = torch.from_numpy(rec).to(dev)
    _lib.check(L.vllt_build_batch_meta(drec.data_ptr(), ctypes.byref(caps), 16, 64, 2,
                                       meta.data_ptr(), _lib.stream_handle()))
    cnt = meta[:16].cpu().numpy()
    assert cnt[7] & 2
    rec_big = np.asarray([9, 3, 1, 1], np.int32)  # more sequences than capacity
    rec_big = np.concatenate([rec_big, np.zeros(40, np.int32)])
    drec_big = torch.from_numpy(rec_big).to(dev)
    _lib.check(L.vllt_build_batch_meta(drec_big.data_ptr(), ctypes.byref(caps), 16, 64,
                                       2, meta.data_ptr(), _lib.stream_handle()))
    assert meta[7].item() & 1


def _meta_fields(L, meta, caps, S, T, R, W):
    import ctypes

    base = meta.data_ptr()

    def field(i, n):
        off = (L.vllt_meta_field(ctypes.c_void_p(base), ctypes.byref(caps), i) - base) // 4
        return meta[off:off + n].cpu().numpy()

    tabs = field(7, caps.max_seqs * caps.max_table_width).reshape(caps.max_seqs, caps.max_table_width)[:S, :W]
    return dict(cnt=field(0, 16), cu_q=field(1, S + 1), cu_rows=field(2, S + 1), ctx=field(3, S), pos=field(4, T),
                slot=field(5, T), rows=field(6, R), tables=tabs)


def test_pooled_batch_meta_matches_the_classic_record(dev):
    """vllt_build_batch_meta_pooled over a persistent device table pool,
    pass after pass of the reference's replays, builds the same metadata as
    vllt_build_batch_meta over the classic record (tables compared on the
    entries each context uses; the pooled builder writes -1 past them)."""
    import ctypes

    from vllt import _lib
    from vllt.runner import StepPacker, tile_positions

    L = _lib.lib()
    for name, bs in (("replay_bench.npz", 16), ("replay_spec.npz", 4)):
        caps = _lib.Caps(16, 1024, 64, 128)
        classic = StepPacker(bs, 512, 261, 512, tile_positions(2))
        pooled = StepPacker(bs, 512, 261, 512, tile_positions(2), pool_slots=32, pool_width=caps.max_table_width)
        pool = torch.full((32, caps.max_table_width), -1, dtype=torch.int32, device=dev)
        n_meta = L.vllt_meta_bytes(ctypes.byref(caps)) // 4
        for seqs, cow, _ in F.replay_steps(name):
            out = F.as_scheduler_output(seqs, cow)
            for seq, s in zip(out.scheduled, seqs):  # one request id per sequence, as the engine's
                seq.seq.request_id = f"b{s['block_ids'][0]}"
            rc, _, _, (S, T, R, W) = classic.pack(out)
            rp, _, _, _ = pooled.pack(out)
            m1 = torch.zeros(n_meta, dtype=torch.int32, device=dev)
            m2 = torch.zeros(n_meta, dtype=torch.int32, device=dev)
            d1, d2 = torch.from_numpy(rc).to(dev), torch.from_numpy(rp).to(dev)
            _lib.check(L.vllt_build_batch_meta(d1.data_ptr(), ctypes.byref(caps), bs, 512, 2, m1.data_ptr(),
                                               _lib.stream_handle()))
            _lib.check(L.vllt_build_batch_meta_pooled(d2.data_ptr(), ctypes.byref(caps), bs, 512, 2,
                                                      pool.data_ptr(), 32, m2.data_ptr(), _lib.stream_handle()))
            a, b = _meta_fields(L, m1, caps, S, T, R, W), _meta_fields(L, m2, caps, S, T, R, W)
            assert a["cnt"][7] == 0 and b["cnt"][7] == 0
            for k in ("cnt", "cu_q", "cu_rows", "ctx", "pos", "slot", "rows"):
                np.testing.assert_array_equal(a[k], b[k], err_msg=k)
            used = -(-a["ctx"] // bs)
            for i in range(S):
                np.testing.assert_array_equal(a["tables"][i, :used[i]], b["tables"][i, :used[i]])
                assert (b["tables"][i, used[i]:] == -1).all()


def test_pooled_batch_meta_flags_bad_updates_without_faulting(dev):
    """An update outside the pool, or a sequence whose row holds an id
    outside [0, num_blocks), raises error bit 1; nothing is written out of
    bounds (the pool's guard row past the 2 rows it is given stays intact)."""
    import ctypes

    from vllt import _lib

    L = _lib.lib()
    caps = _lib.Caps(4, 16, 16, 4)
    pool = torch.full((3, 4), -7, dtype=torch.int32, device=dev)
    meta = torch.zeros(L.vllt_meta_bytes(ctypes.byref(caps)) // 4, dtype=torch.int32, device=dev)

    def build(words):
        rec = torch.from_numpy(np.asarray(words, np.int32)).to(dev)
        _lib.check(L.vllt_build_batch_meta_pooled(rec.data_ptr(), ctypes.byref(caps), 16, 64, 2, pool.data_ptr(), 2,
                                                  meta.data_ptr(), _lib.stream_handle()))
        return int(meta[7].item())

    # S=1 T=3 R=1 W=1 U=1 | start 0 | qlen 3 | count 1 | tokens | slot 1 | update (2, 0, 5): row 2 is outside
    assert build([1, 3, 1, 1, 1, 0, 3, 1, 256, 1, 2, 1, 2, 0, 5]) & 2
    assert pool[2].tolist() == [-7] * 4
    # a valid update, then a row whose entry is out of range
    assert build([1, 3, 1, 1, 1, 0, 3, 1, 256, 1, 2, 1, 1, 0, 5]) == 0
    assert build([1, 3, 1, 1, 1, 0, 3, 1, 256, 1, 2, 0, 0, 0, 99]) & 2


@pytest.mark.parametrize("dtype,H,KV", [("f32", 32, 8), ("bf16", 32, 8), ("bf16", 8, 8), ("bf16", 16, 8),
                                        ("bf16", 64, 8), ("bf16", 12, 6)])
def test_attention_decode_split_k(dev, dtype, H, KV):
    """A pure decode batch with contexts long enough to split across CTAs
    (bf16 / head_dim 128 / block 16 takes the TMA decode kernel)."""
    from vllt.ops import attention_flags, paged_attention_varlen

    rng = np.random.default_rng(11 + H)
    D, bs = 128, 16
    ctxs = [1, 513, 4096, 2000, 17, 1024, 3333]
    qlens = [1] * len(ctxs)
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, bs, qlens, ctxs, np.float32 if dtype == "f32" else "bf16")
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    got = paged_attention_varlen(torch.from_numpy(q).to(dev, tdt), torch.from_numpy(to_lib_layout(ck, bs)).to(dev, tdt),
                                 torch.from_numpy(to_lib_layout(cv, bs)).to(dev, tdt), tab,
                                 np.arange(len(ctxs) + 1), ctxs, 1.0 / np.sqrt(D)).float().cpu().numpy()
    for i, c in enumerate(ctxs):
        slots = A.table_slots(tables[i], bs, c)
        want = A.dense_attention(q[i:i + 1], ck[slots], cv[slots], KV, 1.0 / np.sqrt(D))
        tol = 1e-4 if dtype == "f32" else 2e-2
        np.testing.assert_allclose(got[i:i + 1], want, rtol=tol, atol=tol / 10 if dtype == "f32" else tol)
    assert attention_flags(paged_attention_varlen.last_workspace) == 0


def test_decode_kernel_matches_generic_kernel(dev):
    """The TMA decode kernel and the generic kernel (no workspace) agree."""
    from vllt import _lib
    from vllt.ops import paged_attention_varlen

    rng = np.random.default_rng(5)
    H, KV, D, bs = 32, 8, 128, 16
    ctxs = [4096, 1, 16, 17, 2047, 100]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, bs, [1] * len(ctxs), ctxs, "bf16")
    args = (torch.from_numpy(q).to(dev, torch.bfloat16), torch.from_numpy(to_lib_layout(ck, bs)).to(dev, torch.bfloat16),
            torch.from_numpy(to_lib_layout(cv, bs)).to(dev, torch.bfloat16))
    fast = paged_attention_varlen(*args, tab, np.arange(len(ctxs) + 1), ctxs, 1.0 / np.sqrt(D)).float()
    # generic: pass an explicit NULL workspace through the C ABI
    L = _lib.lib()
    out = torch.empty_like(args[0])
    bt = torch.from_numpy(tab).to(dev)
    cu = torch.arange(len(ctxs) + 1, dtype=torch.int32, device=dev)
    cl = torch.tensor(ctxs, dtype=torch.int32, device=dev)
    _lib.check(L.vllt_paged_attention_varlen(args[0].data_ptr(), args[1].data_ptr(), args[2].data_ptr(), bt.data_ptr(),
                                             tab.shape[1], cu.data_ptr(), cl.data_ptr(), len(ctxs), len(ctxs), 1,
                                             max(ctxs), H, KV, D, bs, args[1].shape[0], float(1 / np.sqrt(D)),
                                             _lib.VLLT_BF16, out.data_ptr(), None, 0, _lib.stream_handle()))
    np.testing.assert_allclose(fast.cpu().numpy(), out.float().cpu().numpy(), rtol=2e-2, atol=2e-2)


def test_attention_prefill_tensor_core_rising_and_falling_scores(dev):
    """Scores that climb by about 10 (log2 units) per 128-key tile make the
    tcgen05 prefill kernel move its running max and rescale O on every tile;
    falling scores keep the first tile's max throughout. Both against the
    float64 oracle on the same bf16 inputs."""
    from vllt.ops import attention_flags, paged_attention_varlen

    rng = np.random.default_rng(11)
    H, KV, D, bs = 32, 8, 128, 16
    qlens, ctxs = [700, 300, 200], [700, 300, 456]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, bs, qlens, ctxs, "bf16")
    u = rng.standard_normal((KV, D))
    u *= np.sqrt(D) / np.linalg.norm(u, axis=1, keepdims=True)
    ramps = [lambda t: 0.005 * t, lambda t: 0.005 * (300 - t), lambda t: 0.004 * t]
    for i, c in enumerate(ctxs):
        for t in range(c):
            slot = tables[i][t // bs] * bs + t % bs
            ck[slot] = u * ramps[i](t) + 0.1 * rng.standard_normal((KV, D))
    cu = np.concatenate([[0], np.cumsum(qlens)])
    for i in range(len(qlens)):
        q[cu[i]:cu[i + 1]] = np.repeat(u, H // KV, axis=0)[None] + 0.1 * rng.standard_normal((qlens[i], H, D))
    r = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy()
    q, ck = r(q), r(ck)
    tq = torch.from_numpy(q).to(dev, torch.bfloat16)
    tk = torch.from_numpy(to_lib_layout(ck, bs)).to(dev, torch.bfloat16)
    tv = torch.from_numpy(to_lib_layout(cv, bs)).to(dev, torch.bfloat16)
    scale = 1.0 / np.sqrt(D)
    got = paged_attention_varlen(tq, tk, tv, tab, cu, ctxs, scale).float().cpu().numpy()
    assert attention_flags(paged_attention_varlen.last_workspace) == 0
    for i, c in enumerate(ctxs):
        slots = A.table_slots(tables[i], bs, c)
        want = A.dense_attention(q[cu[i]:cu[i + 1]], ck[slots], cv[slots], KV, scale)
        np.testing.assert_allclose(got[cu[i]:cu[i + 1]], want, rtol=2e-2, atol=2e-2, err_msg=f"seq {i}")


@pytest.mark.parametrize("H,KV", [(32, 8), (8, 8), (16, 8), (64, 8)])
def test_attention_prefill_tensor_core(dev, H, KV):
    """Multi-token tiles of bf16 / head_dim 128 / block 16 take the tcgen05
    prefill kernel: long prompts (several query and key tiles, diagonal
    masking), chunked prefill over a cached prefix, verify-sized rows and a
    single-token row in the same launch. Checked against the float64 oracle
    and against the generic kernel (no workspace)."""
    from vllt import _lib
    from vllt.ops import attention_flags, paged_attention_varlen

    rng = np.random.default_rng(H + 7)
    D, bs = 128, 16
    qlens = [300, 64, 5, 1, 129, 9]
    ctxs = [300, 1000, 260, 77, 129, 2049]
    q, ck, cv, tables, tab = ragged_batch(rng, H, KV, D, bs, qlens, ctxs, "bf16")
    tq = torch.from_numpy(q).to(dev, torch.bfloat16)
    tk = torch.from_numpy(to_lib_layout(ck, bs)).to(dev, torch.bfloat16)
    tv = torch.from_numpy(to_lib_layout(cv, bs)).to(dev, torch.bfloat16)
    cu = np.concatenate([[0], np.cumsum(qlens)])
    scale = 1.0 / np.sqrt(D)
    got = paged_attention_varlen(tq, tk, tv, tab, cu, ctxs, scale).float().cpu().numpy()
    assert attention_flags(paged_attention_varlen.last_workspace) == 0
    for i, c in enumerate(ctxs):
        slots = A.table_slots(tables[i], bs, c)
        want = A.dense_attention(q[cu[i]:cu[i + 1]], ck[slots], cv[slots], KV, scale)
        np.testing.assert_allclose(got[cu[i]:cu[i + 1]], want, rtol=2e-2, atol=2e-2, err_msg=f"seq {i}")
    # the generic kernel (NULL workspace) on the same batch
    L = _lib.lib()
    out = torch.empty_like(tq)
    bt = torch.from_numpy(tab).to(dev)
    dcu = torch.from_numpy(cu.astype(np.int32)).to(dev)
    dcl = torch.tensor(ctxs, dtype=torch.int32, device=dev)
    _lib.check(L.vllt_paged_attention_varlen(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), bt.data_ptr(), tab.shape[1],
                                             dcu.data_ptr(), dcl.data_ptr(), len(ctxs), int(cu[-1]), max(qlens),
                                             max(ctxs), H, KV, D, bs, tk.shape[0], float(scale), _lib.VLLT_BF16,
                                             out.data_ptr(), None, 0, _lib.stream_handle()))
    np.testing.assert_allclose(got, out.float().cpu().numpy(), rtol=2e-2, atol=2e-2)


def test_decode_benchmark_setup_matches_oracle(dev):
    """The paged-attention decode microbenchmark exactly as bench.py builds it
    (256 sequences, contexts U[1, 4096] from seed 0, 32 / 8 heads, head_dim
    128, bf16, block 16, tables a random permutation of the pool): one new
    token per sequence written through reshape_and_cache, then the TMA decode
    kernel with its 1024-token split-K and merge. Every sequence (all whose
    context crosses a split boundary, and the short ones) is compared with
    the float64 oracle on the same bf16 cache, within the bf16 bar of this
    file (rtol 2e-2, atol 2e-2); the error flag must stay clear."""
    import bench

    s = bench.decode_setup(torch, dev)
    from vllt import _lib

    nbytes = _lib.lib().vllt_attention_workspace_bytes(s["seqs"], s["H"], s["D"], s["max_ctx"])
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(s["q"])
    bench.decode_write(s)
    bench.decode_attend(s, ws, out)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    ctx = s["ctx"].cpu().numpy()
    tables = s["tables"].cpu().numpy()
    q = s["q"].float().cpu().numpy()
    got = out.float().cpu().numpy()
    bs, KV, D = s["bs"], s["KV"], s["D"]
    assert (ctx > 1024).sum() > 150 and (ctx <= 1024).sum() > 30  # split and unsplit sequences
    for i in range(s["seqs"]):
        n = (int(ctx[i]) + bs - 1) // bs
        idx = torch.from_numpy(tables[i, :n].astype(np.int64)).to(dev)
        # [n, KV, bs, D] -> token-major [n * bs, KV, D], first ctx tokens
        k = s["kc"].index_select(0, idx).float().permute(0, 2, 1, 3).reshape(n * bs, KV, D)[:ctx[i]]
        v = s["vc"].index_select(0, idx).float().permute(0, 2, 1, 3).reshape(n * bs, KV, D)[:ctx[i]]
        want = A.dense_attention(q[i:i + 1], k.cpu().numpy(), v.cpu().numpy(), KV, 1.0 / np.sqrt(D))
        np.testing.assert_allclose(got[i:i + 1], want, rtol=2e-2, atol=2e-2, err_msg=f"sequence {i}")
    # the new token landed in the cache at position ctx - 1
    last = ctx - 1
    slot_blk = tables[np.arange(s["seqs"]), last // bs]
    kc_new = s["kc"][torch.from_numpy(slot_blk.astype(np.int64)).to(dev), :, torch.from_numpy(
        (last % bs).astype(np.int64)).to(dev)]
    np.testing.assert_array_equal(kc_new.float().cpu().numpy(), s["knew"].float().cpu().numpy())


def test_decode_wait_expiry_reports_and_recovers(dev):
    """Failure detection of the TMA decode kernel, without a fault: the
    one-shot injection vllt_test_decode_stall arms the stage of table index 3
    for its bytes but issues no copy, with a 2 ms wait limit. Every CTA that
    reads index 3 gives up, sets bit 2 of the workspace flags, lets its other
    copies land and returns: the call itself returns OK. The next call (no
    injection) on the same context is correct with clean flags."""
    from vllt import _lib
    from vllt.ops import attention_flags, paged_attention_varlen

    rng = np.random.default_rng(17)
    S, H, KV, D, bs = 4, 32, 8, 128, 16
    ctx = np.asarray([100, 700, 1500, 50], np.int32)
    nblk = (ctx + bs - 1) // bs
    pool = int(nblk.sum()) + 4
    perm = rng.permutation(pool)
    tab = np.zeros((S, nblk.max()), np.int32)
    o = 0
    for i, n in enumerate(nblk):
        tab[i, :n] = perm[o:o + n]
        o += n
    kc = torch.randn((pool, KV, bs, D), device=dev).to(torch.bfloat16)
    vc = torch.randn((pool, KV, bs, D), device=dev).to(torch.bfloat16)
    q = torch.randn((S, H, D), device=dev).to(torch.bfloat16)
    args = (q, kc, vc, tab, np.arange(S + 1, dtype=np.int32), ctx, 1.0 / np.sqrt(D))
    L = _lib.lib()
    _lib.check(L.vllt_test_decode_stall(3, 2_000_000))
    paged_attention_varlen(*args)
    torch.cuda.synchronize()
    assert attention_flags(paged_attention_varlen.last_workspace) & 4
    out = paged_attention_varlen(*args).float().cpu().numpy()
    assert attention_flags(paged_attention_varlen.last_workspace) == 0
    qh = q.float().cpu().numpy()
    for i in range(S):
        n = int(nblk[i])
        idx = torch.from_numpy(tab[i, :n].astype(np.int64)).to(dev)
        k = kc.index_select(0, idx).float().permute(0, 2, 1, 3).reshape(n * bs, KV, D)[:ctx[i]].cpu().numpy()
        v = vc.index_select(0, idx).float().permute(0, 2, 1, 3).reshape(n * bs, KV, D)[:ctx[i]].cpu().numpy()
        np.testing.assert_allclose(out[i:i + 1], A.dense_attention(qh[i:i + 1], k, v, KV, 1.0 / np.sqrt(D)),
                                   rtol=2e-2, atol=2e-2)


def test_prefix_hash_kernel_matches_hash_block(dev):
    """vllt_prefix_hash_chains: every digest equals the reference's
    hash_block (vllmlite/block.py:34-40) chained as BlockManager chains them,
    for 300 chains of 0 to 40 blocks of 16 tokens, with and without a
    previous block, token ids over the Llama vocabulary."""
    import hashlib

    from vllt.prefix_hash import hash_chains

    def hash_block(prev, toks):  # vllmlite/block.py:34-40
        h = hashlib.blake2b(digest_size=16)
        if prev:
            h.update(prev.encode())
        h.update(b"|")
        h.update(",".join(map(str, toks)).encode())
        return h.hexdigest()

    rng = np.random.default_rng(12)
    chains = []
    for c in range(300):
        n = int(rng.integers(0, 41))
        prev = hash_block(None, [c]) if c % 3 == 0 else None
        chains.append((prev, [int(t) for t in rng.integers(0, 128256, size=16 * n)]))
    got = hash_chains(chains, 16, dev)
    for (prev, toks), hs in zip(chains, got):
        want, p = [], prev
        for b in range(len(toks) // 16):
            p = hash_block(p, toks[16 * b:16 * (b + 1)])
            want.append(p)
        assert hs == want
