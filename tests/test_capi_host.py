"""CPU: libvllt's C ABI entry points, compiled for the host, on the golden fixtures.

The host build of the library (tests/host_build.py build_library_host: the
library's own sources, every kernel on the SIMT emulation) is called through
the same C signatures a reference-side binding uses (vllt/_lib.py SIGNATURES):
  * vllt_paged_attention_varlen on the reference's attention grid
    (tests/golden/attention.npz, made by the reference's paged_attention over
    its own test cases and wider ones): within the reference test's rtol 1e-4
    (vllmlite tests/test_attention.py:57);
  * vllt_paged_attention_varlen_noalloc, the allocation-free entry: bit-identical
    to the workspace entry on every golden case and on ragged batches with
    split-K decode rows and prefill tiles (fp32 and bf16); its device error
    word reads 0, also for an empty batch;
  * vllt_spec_verify on the reference's verify cases: emitted tokens and
    accepted counts;
  * bf16 decode rows (head_dim 128, block 16), which the same entry gives to
    the TMA decode kernel (csrc/decode_kernels.cuh; its tensor-map box loads,
    128-byte swizzle and mbarriers on the emulation's host equivalents):
    against float64 at C3's shape with split-K, and GQA 1 to 8; and the test
    injection of vllt_test_decode_stall, whose armed barrier makes the bounded
    waits expire, set bit 2 and leave the next call clean.
"""

import ctypes as C

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite
from tests.guarded import guarded, ptr

pytestmark = needs_vllmlite


@pytest.fixture
def L(host_library):
    return host_library


def to_block_layout(flat, bs):
    """[slots][n_kv][D] (the reference's cache) -> [blocks][n_kv][bs][D]."""
    s, kv, d = flat.shape
    return np.ascontiguousarray(flat.reshape(s // bs, bs, kv, d).transpose(0, 2, 1, 3))


def attend(L, q, kc, vc, tables, cu, ctx, max_qlen, max_ctx, n_kv, bs, scale, dtype, noalloc=False):
    from vllt import _lib

    T, H, D = q.shape
    S, W = tables.shape
    nb = kc.shape[0]
    out = guarded(np.zeros(q.shape, q.dtype))
    args = [ptr(guarded(q)), ptr(guarded(kc, "start")), ptr(guarded(vc)), ptr(guarded(tables)), W, ptr(guarded(cu)),
            ptr(guarded(ctx, "start")), S, T, max_qlen, max_ctx, H, n_kv, D, bs, nb, scale, dtype, ptr(out)]
    if noalloc:
        flags = guarded(np.full(1, -1, np.int32))
        rc = L.vllt_paged_attention_varlen_noalloc(*args, ptr(flags), None)
        assert rc == 0, L.vllt_last_error()
        assert flags[0] == 0
    else:
        ws = guarded(np.zeros(max(L.vllt_attention_workspace_bytes(S, H, D, max_ctx), 256), np.uint8))
        rc = L.vllt_paged_attention_varlen(*args, ptr(ws), ws.size, None)
        assert rc == 0, L.vllt_last_error()
        assert ws[:4].view(np.int32)[0] == 0  # the workspace header's error word
    return out


def test_paged_attention_entries_on_the_reference_grid(L):
    from vllt import _lib

    n = 0
    for i, inp, want in F.attention_cases():
        bs = inp["block_size"]
        q = inp["q"]
        kc, vc = to_block_layout(inp["cache_k"], bs), to_block_layout(inp["cache_v"], bs)
        tables = np.asarray([inp["block_ids"]], np.int32)
        cu = np.array([0, q.shape[0]], np.int32)
        ctx = np.array([inp["ctx"]], np.int32)
        a = attend(L, q, kc, vc, tables, cu, ctx, q.shape[0], inp["ctx"], inp["n_kv"], bs, inp["scale"], _lib.VLLT_F32)
        np.testing.assert_allclose(a, want, rtol=1e-4, atol=1e-5, err_msg=f"case {i}")
        b = attend(L, q, kc, vc, tables, cu, ctx, q.shape[0], inp["ctx"], inp["n_kv"], bs, inp["scale"], _lib.VLLT_F32,
                   noalloc=True)
        np.testing.assert_array_equal(a, b)
        n += 1
    assert n == 39


def _bf16(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("qlens,ctxs", [([1, 1, 1], [700, 1300, 5]), ([12, 1, 40], [12, 600, 90])])
def test_noalloc_entry_is_bit_identical_to_the_workspace_entry(L, bf16, qlens, ctxs):
    """Ragged batches: single-query passes over more than 512 keys split the
    context (the partials live in the static scratch), mixed passes run
    prefill tiles; the two entries run the same kernels and agree bit for bit."""
    from vllt import _lib

    rng = np.random.default_rng(sum(ctxs) + bf16)
    H, n_kv, D, bs = 8, 4, 48, 16
    W = max(-(-c // bs) for c in ctxs)
    nb = sum(-(-c // bs) for c in ctxs) + 3
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.full((len(ctxs), W), -1, np.int32)
    o = 0
    for s, c in enumerate(ctxs):
        n = -(-c // bs)
        tables[s, :n] = perm[o:o + n]
        o += n
    T = sum(qlens)
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    kc = rng.standard_normal((nb, n_kv, bs, D)).astype(np.float32)
    vc = rng.standard_normal((nb, n_kv, bs, D)).astype(np.float32)
    dtype = _lib.VLLT_F32
    if bf16:
        q, kc, vc = _bf16(q), _bf16(kc), _bf16(vc)
        dtype = _lib.VLLT_BF16
    cu = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    ctx = np.asarray(ctxs, np.int32)
    args = (q, kc, vc, tables, cu, ctx, max(qlens), max(ctxs), n_kv, bs, 1 / np.sqrt(D), dtype)
    a = attend(L, *args)
    b = attend(L, *args, noalloc=True)
    np.testing.assert_array_equal(a, b)
    assert (a != 0).any()


def test_noalloc_empty_batch_writes_a_clean_flag(L):
    flags = guarded(np.full(1, -1, np.int32))
    assert L.vllt_paged_attention_varlen_noalloc(None, None, None, None, 1, None, None, 0, 0, 0, 0, 8, 4, 48, 16, 64,
                                                 0.1, 0, None, ptr(flags), None) == 0
    assert flags[0] == 0


def test_spec_verify_entry_on_the_reference_cases(L):
    z = F.load("sampling.npz")
    ks, lg = z["verify_k"], z["verify_logits"]
    S, V = len(ks), lg.shape[1]
    cu = np.concatenate([[0], np.cumsum(ks + 1)]).astype(np.int32)
    doff = np.concatenate([[0], np.cumsum(ks)[:-1]]).astype(np.int32)
    out = guarded(np.full(int(cu[-1]), -7, np.int32))
    acc = guarded(np.full(S, -7, np.int32))
    assert L.vllt_spec_verify(ptr(guarded(lg.astype(np.float32))), V, V, ptr(guarded(cu)), int(cu[-1]),
                              ptr(guarded(z["verify_drafts"].astype(np.int32))), ptr(guarded(doff)), S, ptr(out),
                              ptr(acc), None) == 0
    assert acc.tolist() == z["verify_accepted"].tolist()
    to = 0
    for s in range(S):
        nt = int(z["verify_ntok"][s])
        assert out[cu[s]:cu[s] + nt].tolist() == z["verify_tokens"][to:to + nt].tolist()
        to += nt


# ---- the TMA decode kernel (csrc/decode_kernels.cuh) through the same entry ---------

def _decode_case(rng, ctxs, H, n_kv, spare=5):
    """bf16 single-query batch over the [block][kv head][16][128] cache."""
    D, bs = 128, 16
    S, W = len(ctxs), max(-(-c // bs) for c in ctxs)
    nb = sum(-(-c // bs) for c in ctxs) + spare
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.full((S, W), -1, np.int32)
    o = 0
    for s, c in enumerate(ctxs):
        n = -(-c // bs)
        tables[s, :n] = perm[o:o + n]
        o += n
    q = _bf16(rng.standard_normal((S, H, D)))
    kc = _bf16(rng.standard_normal((nb, n_kv, bs, D)))
    vc = _bf16(rng.standard_normal((nb, n_kv, bs, D)))
    return q, kc, vc, tables, nb


def _f(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def _decode_want(q, kc, vc, tables, ctxs, n_kv, scale):
    from oracle.attention import dense_attention

    out = []
    for s, c in enumerate(ctxs):
        blocks = tables[s, :-(-c // 16)]
        k = _f(kc[blocks]).transpose(0, 2, 1, 3).reshape(-1, n_kv, 128)[:c]
        v = _f(vc[blocks]).transpose(0, 2, 1, 3).reshape(-1, n_kv, 128)[:c]
        out.append(dense_attention(_f(q[s:s + 1]), k, v, n_kv, scale)[0])
    return np.stack(out)


@pytest.mark.parametrize("H,n_kv,ctxs", [
    (32, 8, [4096, 1, 2047, 16, 17, 1025, 3000, 100, 4000, 63, 640, 2500]),   # C3's shape, 4 splits
    (8, 8, [33, 700]), (16, 8, [1300, 5]), (64, 8, [260, 1100]),             # GQA 1, 2, 8
])
@pytest.mark.parametrize("seed", [0, 0x5EED])
def test_tma_decode_kernel_against_float64(L, H, n_kv, ctxs, seed):
    """bf16 decode rows (head_dim 128, block 16) go to the TMA decode kernel:
    tensor-map box loads with the 128-byte swizzle into per-warp rings guarded
    by mbarriers, split-K over 64-block chunks with the merge kernel. Against a
    float64 restatement of the reference's attention, within one bf16
    rounding of the output; the error word stays 0."""
    from vllt import _lib

    rng = np.random.default_rng(sum(ctxs) + H)
    q, kc, vc, tables, nb = _decode_case(rng, ctxs, H, n_kv)
    S = len(ctxs)
    cu = np.arange(S + 1, dtype=np.int32)
    ctx = np.asarray(ctxs, np.int32)
    scale = 1 / np.sqrt(128)
    L.vllt_host_schedule_seed.argtypes = [C.c_uint64]
    L.vllt_host_schedule_seed(seed)  # nonzero: the shuffled schedule
    try:
        out = attend(L, q, kc, vc, tables, cu, ctx, 1, max(ctxs), n_kv, 16, scale, _lib.VLLT_BF16)
    finally:
        L.vllt_host_schedule_seed(0)
    want = _decode_want(q, kc, vc, tables, ctxs, n_kv, scale)
    np.testing.assert_allclose(_f(out), want, rtol=2.0 ** -7, atol=2e-3)


def test_decode_stall_injection_reports_and_recovers(L):
    """vllt_test_decode_stall arms one stage's mbarrier for its bytes without
    issuing the copies: every CTA reading that table index sees its bounded
    wait expire, sets bit 2 of the error word, drains its other copies and
    returns; the next call is clean and equals a normal run."""
    from vllt import _lib

    rng = np.random.default_rng(11)
    ctxs = [300, 90]
    q, kc, vc, tables, nb = _decode_case(rng, ctxs, 32, 8)
    S = len(ctxs)
    cu = np.arange(S + 1, dtype=np.int32)
    ctx = np.asarray(ctxs, np.int32)
    args = (q, kc, vc, tables, cu, ctx, 1, max(ctxs), 8, 16, 1 / np.sqrt(128), _lib.VLLT_BF16)
    clean = attend(L, *args)
    assert L.vllt_test_decode_stall(3, 2_000_000) == 0  # table index 3, 2 ms waits
    T, H, D = q.shape
    W = tables.shape[1]
    out = guarded(np.zeros(q.shape, q.dtype))
    ws = guarded(np.zeros(max(L.vllt_attention_workspace_bytes(S, H, D, max(ctxs)), 256), np.uint8))
    assert L.vllt_paged_attention_varlen(ptr(guarded(q)), ptr(guarded(kc)), ptr(guarded(vc)), ptr(guarded(tables)), W,
                                         ptr(guarded(cu)), ptr(guarded(ctx)), S, T, 1, max(ctxs), H, 8, D, 16, nb,
                                         1 / np.sqrt(128), _lib.VLLT_BF16, ptr(out), ptr(ws), ws.size, None) == 0
    assert ws[:4].view(np.int32)[0] & 4
    again = attend(L, *args)  # asserts a clean error word
    np.testing.assert_array_equal(again, clean)
