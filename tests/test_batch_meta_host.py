"""CPU: the device batch flatten's arithmetic against the reference.

build_meta_kernel (csrc/batch_meta_kernels.cuh) keeps its per-item
arithmetic in csrc/meta_items.cuh. Every test runs twice: on
tests/meta_host.cpp, which runs the kernel's phases one after another with
those functions compiled for the host, and on the kernel's own code under the
host SIMT emulation (one CTA of 1024 fibers, tests/kernels_host.cpp), with
the emulation's default schedule and with a seeded shuffle after every
barrier. On every pass of the
reference's replays (the bench model with chunked prefill; speculative k = 4
with the prefix cache, block 4) the metadata it builds from the packed step
record (classic, and pooled with a persistent table pool) must equal the
reference's ModelRunner.execute flatten (vllmlite/runner.py:66-90, restated by
oracle.runner.flatten): positions, write slots, logit rows, cumulative
lengths; and the two record forms must build the same metadata. Bad records
raise the kernel's error bits without touching memory they do not own.
"""

import ctypes

import numpy as np
import pytest

from oracle import runner as OR
from tests import fixtures as F


ARGS = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 8 + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                                 ctypes.c_int]


class _Kernel:
    """build_meta_kernel's own code on the host SIMT emulation (one CTA of
    1024 fibers), behind the phase harness's entry point."""

    def __init__(self, lib):
        self.lib = lib

    def build_meta_host(self, *a):
        guard = [a[0], a[1]]  # keep the ctypes call's buffers as given
        rc = self.lib.run_build_meta(*a)
        assert rc == 0, "the CTA's threads waited on barriers that cannot complete"
        del guard
        # the kernel reports through the counters' error word, as on the device
        meta_ptr = a[10]
        return int(np.ctypeslib.as_array((ctypes.c_int32 * 16).from_address(meta_ptr))[7])


@pytest.fixture(scope="module", params=["phases", "kernel", "kernel-shuffled"])
def meta_host(request, tmp_path_factory):
    """The builder run as its phases one after another (tests/meta_host.cpp),
    or as the kernel itself on the host SIMT emulation (tests/kernels_host.cpp)."""
    from tests.host_build import build_harness

    if request.param == "phases":
        lib = build_harness("meta_host", str(tmp_path_factory.mktemp("meta")))
        if lib is None:
            pytest.skip("g++ is not available")
        lib.build_meta_host.argtypes = ARGS
        return lib
    lib = build_harness("kernels_host", str(tmp_path_factory.mktemp("meta_kernel")))
    if lib is None:
        pytest.skip("g++ is not available")
    lib.run_build_meta.argtypes = ARGS
    lib.set_schedule_seed.argtypes = [ctypes.c_uint64]
    lib.set_schedule_seed(0x5DEECE66D if request.param == "kernel-shuffled" else 0)
    return _Kernel(lib)


def build(host, rec, caps, bs, nb, qp, pool=None, tsrc=None, vocab=261):
    from vllt import _lib

    L = _lib.lib()
    words = L.vllt_meta_bytes(ctypes.byref(caps)) // 4
    meta = np.full(words, -7, np.int32)
    rec = np.ascontiguousarray(rec, np.int32)
    err = host.build_meta_host(rec.ctypes.data, pool.ctypes.data if pool is not None else None,
                               pool.shape[0] if pool is not None else 0, caps.max_seqs, caps.max_tokens,
                               caps.max_rows, caps.max_table_width, bs, nb, qp, meta.ctypes.data,
                               tsrc.ctypes.data if tsrc is not None else None,
                               tsrc.size if tsrc is not None else 0, vocab)
    base = meta.ctypes.data

    def field(i, n):  # offsets from the library's own layout function (host arithmetic only)
        off = (L.vllt_meta_field(ctypes.c_void_p(base), ctypes.byref(caps), i) - base) // 4
        return meta[off:off + n]

    return err, meta, field


@pytest.mark.parametrize("name,bs", [("replay_bench.npz", 16), ("replay_spec.npz", 4)])
def test_kernel_arithmetic_builds_the_reference_flatten(meta_host, name, bs):
    from vllt import _lib
    from vllt.runner import StepPacker, tile_positions

    qp = tile_positions(2)
    caps = _lib.Caps(16, 1024, 64, 128)
    classic = StepPacker(bs, 512, 261, 512, qp)
    pooled = StepPacker(bs, 512, 261, 512, qp, pool_slots=32, pool_width=caps.max_table_width)
    pool = np.full((32, caps.max_table_width), -1, np.int32)
    n = 0
    for seqs, cow, _ in F.replay_steps(name):
        out = F.as_scheduler_output(seqs, cow)
        for item, s in zip(out.scheduled, seqs):  # one request id per sequence, as the engine's
            item.seq.request_id = f"b{s['block_ids'][0]}"
        rc, bounds, rows, (S, T, R, W) = classic.pack(out)
        rp = pooled.pack(out)[0]
        e1, m1, f1 = build(meta_host, rc, caps, bs, 512, qp)
        e2, m2, f2 = build(meta_host, rp, caps, bs, 512, qp, pool)
        assert e1 == 0 and e2 == 0
        tok, pos, smeta, last, orows = OR.flatten(seqs, bs)
        for f in (f1, f2):
            cnt = f(0, 16)
            assert cnt[:4].tolist() == [S, T, R, W] and cnt[7] == 0
            assert cnt[4] == bounds.decode_seqs and cnt[5] == bounds.tiles and cnt[6] == bounds.max_ctx
            assert f(1, S + 1).tolist() == [0] + np.cumsum([s["n"] for s in seqs]).tolist()
            assert f(4, T).tolist() == pos.tolist()
            assert f(5, T).tolist() == np.concatenate([m[2] for m in smeta]).tolist()
            assert f(6, R).tolist() == last.tolist()
            assert f(3, S).tolist() == [s["start"] + s["n"] for s in seqs]
        # both record forms: the same metadata on every entry a pass reads
        for i in (0, 1, 2, 3, 4, 5, 6):
            np.testing.assert_array_equal(f1(i, 16 if i == 0 else {1: S + 1, 2: S + 1, 3: S, 4: T, 5: T, 6: R}[i]),
                                          f2(i, 16 if i == 0 else {1: S + 1, 2: S + 1, 3: S, 4: T, 5: T, 6: R}[i]))
        n += 1
    assert n > 10


def test_kernel_arithmetic_flags_bad_records(meta_host):
    """The checks of build_meta_kernel on bad step records: an unknown block
    id (bit 1, its slot -1, the step still built), a capacity overflow (bit 0,
    counters zeroed), fields the runner could not index with (bit 1, counters
    zeroed), a pool update outside the pool (bit 1, nothing written)."""
    from vllt import _lib

    caps = _lib.Caps(4, 16, 16, 4)
    # S=1 T=3 R=1 W=1 | start 0 | qlen 3 | count 1 | tokens | block 777 >= num_blocks
    err, meta, f = build(meta_host, [1, 3, 1, 1, 0, 3, 1, 256, 1, 2, 777], caps, 16, 64, 8)
    assert err & 2 and f(5, 3).tolist() == [-1, -1, -1] and f(0, 16)[0] == 1
    err, meta, f = build(meta_host, [9, 3, 1, 1] + [0] * 40, caps, 16, 64, 8)  # more sequences than capacity
    assert err == 1 and f(0, 16)[:7].tolist() == [0] * 7
    err, meta, f = build(meta_host, [1, 3, 1, 1, 0, 3, 4, 256, 1, 2, 5], caps, 16, 64, 8)  # count > qlen
    assert err & 2 and f(0, 16)[0] == 0
    pool = np.full((3, 4), -7, np.int32)
    pooled_bad = [1, 3, 1, 1, 1, 0, 3, 1, 256, 1, 2, 1, 2, 0, 5]  # update (2, 0, 5): row 2 of a 2-row pool
    err, meta, f = build(meta_host, pooled_bad, caps, 16, 64, 8, pool[:2])
    assert err & 2 and pool[2].tolist() == [-7] * 4


def test_kernel_arithmetic_resolves_token_references(meta_host):
    """Record token ids t < 0 read entry -t - 1 of the previous pass's picks
    (the token source); a reference outside the source, a resolved id outside
    the vocabulary, or a negative id without a source embeds token 0 and sets
    bit 1 (the step stays runnable); ids >= vocab are flagged the same way."""
    from vllt import _lib

    caps = _lib.Caps(4, 16, 16, 4)
    picks = np.array([7, 250, 3, 300, -1], np.int32)  # entries 3 and 4 are not tokens of a 261 vocabulary
    # two decode sequences: tokens -(1 + 1) -> picks[1] = 250, 5 -> 5
    rec = [2, 2, 2, 1, 0, 4, 1, 1, 1, 1, -2, 5, 1, 2]
    err, meta, f = build(meta_host, rec, caps, 16, 64, 8, tsrc=picks)
    assert err == 0 and f(8, 2).tolist() == [250, 5]
    for bad_tok in (-4, -5, -6, 261):  # picks[3] = 300, picks[4] = -1, beyond the source, beyond the vocabulary
        err, meta, f = build(meta_host, [2, 2, 2, 1, 0, 4, 1, 1, 1, 1, bad_tok, 5, 1, 2], caps, 16, 64, 8,
                             tsrc=picks)
        assert err == 2 and f(8, 2).tolist() == [0, 5] and f(0, 16)[0] == 2
    err, meta, f = build(meta_host, rec, caps, 16, 64, 8)  # no source
    assert err == 2 and f(8, 2).tolist() == [0, 5]


def test_a_runnable_error_leaves_every_token_built(meta_host):
    """A bad block id is flagged in phase 2 while the step stays runnable:
    every one of the step's tokens (here 100, spread over four warps) still
    gets its position, token and slot. The stop flag that every thread reads
    after phase 1 is a separate word from the phase-2/3 flags, so a warp
    that reads it late cannot see a later phase's error and leave early."""
    from vllt import _lib

    caps = _lib.Caps(4, 128, 16, 8)
    toks = list(range(100))
    rec = [1, 100, 1, 7, 0, 100, 1] + toks + [3, 4, 5, 777, 6, 7, 8]  # block 3 of 7 is unknown
    err, meta, f = build(meta_host, rec, caps, 16, 64, 8)
    assert err == 2 and f(0, 16)[0] == 1
    assert f(4, 100).tolist() == list(range(100)) and f(8, 100).tolist() == toks
    slots = f(5, 100)
    assert slots[48:64].tolist() == [-1] * 16 and slots[:48].tolist() == [3 * 16 + i for i in range(16)] + \
        [4 * 16 + i for i in range(16)] + [5 * 16 + i for i in range(16)]
    assert slots[64:].tolist() == [6 * 16 + i for i in range(16)] + [7 * 16 + i for i in range(16)] + \
        [8 * 16 + i for i in range(4)]
