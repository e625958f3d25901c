"""CPU: device-resident block tables (pooled step records) against the classic record.

The runner keeps every live sequence's block table in a persistent device pool
and uploads per pass only the (row, index, block id) entries that changed
(include/vllt.h, "pooled record"). Here the unmodified reference engine
(Scheduler, BlockManager with prefix caching, copy-on-write, preemption, the
n-gram proposer) drives a runner that packs every pass both ways; the pooled
record's updates are applied to a host copy of the pool twice: by a NumPy
restatement of build_meta_kernel's phases 0 and 2, and by the kernel's own
per-item code (csrc/meta_items.cuh, compiled for the host by g++). The tables
read back through each sequence's row must equal the classic record's tables
bit for bit, on the 48-request mixed-length (C1) and shared-prefix (C2)
benchmarks, the 512-request Llama-shaped workload (C4), and small runs that
force preemption and speculative rejections. The pooled record must also
carry O(S + T + changed entries) words.
"""

import numpy as np
import pytest

from tests.conftest import needs_vllmlite

pytestmark = needs_vllmlite


HOST = {}  # the host-compiled build_meta_kernel pool phases (tests/meta_host.cpp), when g++ exists


@pytest.fixture(autouse=True, scope="module")
def _host_pool_phases(tmp_path_factory):
    import ctypes

    from tests.host_build import build_harness

    lib = build_harness("meta_host", str(tmp_path_factory.mktemp("tp")))
    if lib is not None:
        lib.apply_pooled_host.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
        HOST["lib"] = lib
    yield
    HOST.clear()


def apply_pooled_kernel_code(pool, rec, bs, num_blocks):
    """The same phases with the kernel's own per-item code (pool_update /
    pool_entry of csrc/meta_items.cuh) compiled for the host."""
    S, W = int(rec[0]), int(rec[3])
    rec = np.ascontiguousarray(rec, np.int32)
    out = np.zeros((S, W), np.int32)
    err = HOST["lib"].apply_pooled_host(rec.ctypes.data, pool.ctypes.data, pool.shape[0], pool.shape[1], bs,
                                        num_blocks, out.ctypes.data)
    return out, err


def apply_pooled(pool, f, bs, num_blocks):
    """Phases 0 and 2 of build_meta_kernel for a pooled record: apply the
    updates, then the tables each sequence reads ([S][W], -1 past the blocks
    its context uses). Returns (tables, error flag)."""
    err = 0
    slots, width = pool.shape
    for sl, j, blk in f["updates"]:
        if 0 <= sl < slots and 0 <= j < width:
            pool[sl, j] = blk
        else:
            err |= 2
    S, W = f["S"], f["W"]
    out = np.full((S, W), -1, np.int64)
    ctx = f["start"].astype(np.int64) + f["qlen"]
    for s in range(S):
        used = -(-int(ctx[s]) // bs)
        sl = int(f["slot"][s])
        if 0 <= sl < slots:
            out[s, :used] = pool[sl, :used]
        bad = (out[s, :used] < 0) | (out[s, :used] >= num_blocks)
        if bad.any():
            err |= 2
            out[s, :used][bad] = -1
    return out, err


class PackingRunner:
    """A ModelRunner (vllmlite/runner.py:19-32) that packs each pass as the
    classic and the pooled record, checks that they describe the same tables,
    and returns deterministic pseudo-random logits (so speculative drafts are
    sometimes rejected)."""

    continue_prompts = False  # logits that continue each prompt periodically (drafts get accepted)

    def __init__(self, model_cfg, cache_cfg, vocab_out=64):
        from vllt.runner import StepPacker

        self.model_cfg = model_cfg
        self.bs, self.nb = cache_cfg.block_size, cache_cfg.num_blocks
        width = -(-model_cfg.max_seq_len // self.bs) + 8
        args = (self.bs, self.nb, model_cfg.vocab_size, model_cfg.max_seq_len + 16, 8)
        self.classic = StepPacker(*args)
        self.pooled = StepPacker(*args, pool_slots=2 * 512, pool_width=width)
        self.pool = np.full((2 * 512, width), -1, np.int32)
        self.pool_k = self.pool.copy()  # the pool as the kernel's host-compiled code leaves it
        self.vocab_out = vocab_out
        self.words = {"classic": 0, "pooled": 0}
        self.passes = self.updates = self.kernel_code_passes = 0

    @property
    def vocab_size(self):
        return self.model_cfg.vocab_size

    @property
    def cache_bytes(self):
        return 0

    def execute(self, out):
        rc, _, rows, (S, T, R, W) = self.classic.pack(out)
        rp, _, rows_p, dims_p = self.pooled.pack(out)
        assert rows_p == rows and dims_p == (S, T, R, W)
        fc, fp = self.classic.fields(rc), self.pooled.fields(rp)
        for k in ("start", "qlen", "count", "tokens"):
            np.testing.assert_array_equal(fc[k], fp[k])
        got, err = apply_pooled(self.pool, fp, self.bs, self.nb)
        assert err == 0
        if "lib" in HOST:
            got_k, err_k = apply_pooled_kernel_code(self.pool_k, rp, self.bs, self.nb)
            assert err_k == 0
            np.testing.assert_array_equal(got_k, got)
            self.kernel_code_passes += 1
        ctx = fc["start"].astype(np.int64) + fc["qlen"]
        for s in range(S):
            used = -(-int(ctx[s]) // self.bs)
            np.testing.assert_array_equal(got[s, :used], fc["tables"][s, :used])
        # pooled words: header, per-sequence fields, tokens, slots and only the changed entries
        assert rp.size == 5 + 4 * S + T + 3 * fp["U"]
        self.words["classic"] += rc.size
        self.words["pooled"] += rp.size
        self.passes += 1
        self.updates += fp["U"]
        V = self.vocab_size if self.continue_prompts else self.vocab_out
        logits = np.zeros((R, V), np.float32)
        for i, item in enumerate(out.scheduled):
            r0, n = rows[i]
            p = item.seq.prompt_token_ids
            for j in range(n):
                pos = item.start_pos + item.num_tokens - n + j
                if self.continue_prompts:  # the prompt again, except every 11th position
                    tok = p[(pos + 1) % len(p)] if pos % 11 else 1
                else:
                    tok = (pos * 7 + len(p) * 13) % V
                logits[r0 + j, tok] = 1.0
        return logits, rows


def run_engine(cfg, reqs, spec_k=0):
    import vllmlite.engine as E

    orig = E.NumpyRunner
    E.NumpyRunner = PackingRunner
    try:
        eng = E.LLMEngine(cfg, None, spec_k)
    finally:
        E.NumpyRunner = orig
    for rid, ids, p in reqs:
        eng.add_request(params=p, request_id=rid, prompt_token_ids=ids)
    while eng.has_work:
        eng.step()
    return eng


def engine_cfg(n_layers=6, vocab=261, max_len=512, bs=16, nb=512, max_seqs=16, budget=1024, prefix=False):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    mc = ModelConfig(n_layers=n_layers, n_heads=8, n_kv_heads=4, d_model=384, d_ff=1024, vocab_size=vocab,
                     max_seq_len=max_len)
    return EngineConfig(model=mc, cache=CacheConfig(block_size=bs, num_blocks=nb, enable_prefix_caching=prefix),
                        scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget))


def check(eng, ratio):
    run = eng.runner
    assert run.passes > 10 and run.updates > 0
    assert run.kernel_code_passes == (run.passes if "lib" in HOST else 0)
    assert run.words["pooled"] * ratio < run.words["classic"], run.words
    return run


def test_pooled_tables_on_the_mixed_length_benchmark():
    from vllt.workloads import mixed_workload

    check(run_engine(engine_cfg(), mixed_workload(48, 0, 0)), 1.2)


def test_pooled_tables_on_the_shared_prefix_benchmark():
    from vllt.workloads import mixed_workload

    eng = run_engine(engine_cfg(max_len=768, nb=768, prefix=True), mixed_workload(48, 0, 256))
    check(eng, 2)
    assert eng.scheduler.blocks.allocator.hits > 0


def test_pooled_tables_on_the_llama_workload():
    """C4: 512 requests, budget 8192, 16-token blocks; the classic record
    carries 512 x W table words per decode pass, the pooled one a few."""
    from vllt.workloads import llama_workload

    cfg = engine_cfg(vocab=128256, max_len=9216, nb=40000, max_seqs=512, budget=8192)
    run = check(run_engine(cfg, llama_workload(512, seed=0)), 20)
    assert run.passes > 500


@pytest.mark.parametrize("prefix", [False, True])
def test_pooled_tables_under_preemption(prefix):
    """Few blocks: sequences are preempted (their table replaced by a new,
    empty one) and later rebuilt, with and without prefix reuse."""
    from vllt.workloads import mixed_workload

    eng = run_engine(engine_cfg(bs=4, nb=96, max_seqs=8, budget=64, prefix=prefix), mixed_workload(12, 3, 0))
    check(eng, 1.0)
    assert eng.scheduler.total_preemptions > 0


def test_pooled_tables_with_speculation_and_copy_on_write():
    """n-gram drafts (some rejected, so tables hold blocks past num_filled)
    over shared prompt prefixes in 4-token blocks with prefix caching."""
    from vllmlite.sequence import SamplingParams

    from vllt.workloads import periodic_lengths

    reqs = []
    for i, (ids, _) in enumerate(periodic_lengths(16, seed=2, max_tokens=40)):
        reqs.append((f"p{i}", ids[:30] if i % 2 else ids[:61], SamplingParams(max_tokens=40, temperature=0.0,
                                                                               ignore_eos=True)))
    reqs += [(f"d{i}", list(reqs[0][1]), SamplingParams(max_tokens=24, temperature=0.0, ignore_eos=True))
             for i in range(3)]
    PackingRunner.continue_prompts = True
    try:
        eng = run_engine(engine_cfg(bs=4, nb=1024, max_seqs=8, budget=256, prefix=True), reqs, spec_k=4)
    finally:
        PackingRunner.continue_prompts = False
    check(eng, 1.0)
    assert eng.spec.proposed > eng.spec.accepted > 0
    assert eng.scheduler.blocks.allocator.hits > 0


def test_pool_rows_are_reused_least_recently_scheduled_first():
    """With fewer rows than sequences over time, a new sequence takes the row
    of the sequence scheduled longest ago, and a row is never taken from a
    sequence of the same pass."""
    from types import SimpleNamespace as NS

    from vllt.runner import StepPacker

    pk = StepPacker(4, 64, 100, 64, 8, pool_slots=2, pool_width=8)

    def item(rid, blocks, start=0, n=3):
        seq = NS(request_id=rid, token_ids=list(range(start + n)), draft_token_ids=[], table=NS(block_ids=blocks))
        return NS(seq=seq, start_pos=start, num_tokens=n)

    a, b, c = item("a", [1]), item("b", [2]), item("c", [3])
    f = pk.fields(pk.pack(NS(scheduled=[a, b], cow=[]))[0])
    assert sorted(f["slot"].tolist()) == [0, 1] and f["U"] == 2
    f = pk.fields(pk.pack(NS(scheduled=[b], cow=[]))[0])
    assert f["U"] == 0  # nothing changed for b
    slot_b = int(f["slot"][0])
    f = pk.fields(pk.pack(NS(scheduled=[c, b], cow=[]))[0])
    assert int(f["slot"][0]) == 1 - slot_b  # a's row, the least recently scheduled
    assert f["updates"].tolist() == [[1 - slot_b, 0, 3]]
    with pytest.raises(ValueError):
        pk.pack(NS(scheduled=[a, b, c], cow=[]))  # three sequences, two rows


def test_copy_on_write_replacement_is_uploaded():
    """BlockManager.append_slots replaces a shared, partly filled block in
    place (block_manager.py:77-85): the table object stays the same and the
    entry at num_filled // block_size changes value. The pooled record must
    carry exactly that entry (and any appended block), and a table replaced by
    a new object (preemption) is compared entry by entry."""
    from types import SimpleNamespace as NS

    from vllt.runner import StepPacker

    pk = StepPacker(16, 64, 100, 256, 8, pool_slots=4, pool_width=8)
    pool = np.full((4, 8), -1, np.int32)
    tbl = NS(block_ids=[5, 6])
    seq = NS(request_id="x", token_ids=list(range(40)), draft_token_ids=[], table=tbl)

    def step(start, n):
        rec = pk.pack(NS(scheduled=[NS(seq=seq, start_pos=start, num_tokens=n)], cow=[]))[0]
        f = pk.fields(rec)
        tables, err = apply_pooled(pool, f, 16, 64)
        assert err == 0
        return f["updates"].tolist(), tables[0].tolist()

    ups, tab = step(0, 20)
    assert ups == [[0, 0, 5], [0, 1, 6]] and tab == [5, 6]
    tbl.block_ids[1] = 9  # copy-on-write of the half-filled block 6 -> 9
    ups, tab = step(20, 1)
    assert ups == [[0, 1, 9]] and tab == [5, 9]
    tbl.block_ids.append(11)  # decode crosses into a new block
    ups, tab = step(32, 1)
    assert ups == [[0, 2, 11]] and tab == [5, 9, 11]
    seq.table = NS(block_ids=[5, 7, 11])  # a new table object: compared from entry 0
    ups, tab = step(0, 33)
    assert ups == [[0, 1, 7]] and tab == [5, 7, 11]


def test_pooled_packing_rejects_what_the_reference_cannot_index():
    from types import SimpleNamespace as NS

    from vllt.runner import StepPacker

    pk = StepPacker(16, 64, 100, 256, 8, pool_slots=4, pool_width=4)

    def pack(blocks, start=0, n=3, rid="y"):
        seq = NS(request_id=rid, token_ids=list(range(start + n)), draft_token_ids=[], table=NS(block_ids=blocks))
        return pk.pack(NS(scheduled=[NS(seq=seq, start_pos=start, num_tokens=n)], cow=[]))

    with pytest.raises(IndexError):
        pack([64])  # block id beyond num_blocks
    with pytest.raises(IndexError):
        pack([-1], rid="z")  # -1 equals an unknown mirror entry: still refused
    with pytest.raises(IndexError):
        pack([1], n=20, rid="w")  # table too short for the context
    with pytest.raises(ValueError):
        pack([1, 2, 3, 4, 5], rid="v")  # wider than the pool


@pytest.mark.parametrize("seed", range(6))
def test_pooled_tables_under_random_table_histories(seed):
    """Random pass sequences without the reference scheduler: sequences grow
    block by block, have the block being written replaced (copy-on-write),
    get a new empty table and are rebuilt (preemption), retire, and new ones
    arrive, with fewer pool rows than sequences over time. After every pass
    the tables read through the pool (both restatements of the kernel's
    phases) equal the classic record's."""
    from types import SimpleNamespace as NS

    from vllt.runner import StepPacker

    rng = np.random.default_rng(seed)
    bs, nb, width, rows = 4, 4096, 40, 12
    classic = StepPacker(bs, nb, 100, 160, 8)
    pooled = StepPacker(bs, nb, 100, 160, 8, pool_slots=rows, pool_width=width)
    pool = np.full((rows, width), -1, np.int32)
    pool_k = pool.copy()
    live, next_id = [], 0
    for step in range(120):
        while len(live) < 8 and rng.random() < 0.5:  # arrivals
            live.append(NS(request_id=f"q{next_id}", table=NS(block_ids=[]), filled=0, draft_token_ids=[]))
            next_id += 1
        sched = []
        for seq in list(live):
            r = rng.random()
            if r < 0.05:  # retire
                live.remove(seq)
                continue
            if r < 0.12:  # preempted: a new empty table, recomputed from position 0
                seq.table, seq.filled = NS(block_ids=[]), 0
            if rng.random() < 0.3:
                continue  # not scheduled this pass
            n = int(rng.integers(1, 9))
            if seq.filled + n > 150:
                live.remove(seq)
                continue
            ids = seq.table.block_ids
            if seq.filled % bs and ids and rng.random() < 0.3:  # copy-on-write of the block being written
                ids[seq.filled // bs] = int(rng.integers(0, nb))
            while len(ids) * bs < seq.filled + n:
                ids.append(int(rng.integers(0, nb)))
            seq.token_ids = [1] * (seq.filled + n)
            sched.append(NS(seq=seq, start_pos=seq.filled, num_tokens=n))
            seq.filled += n
        if not sched:
            continue
        out = NS(scheduled=sched, cow=[])
        rc = classic.pack(out)[0]
        rp = pooled.pack(out)[0]
        fc, fp = classic.fields(rc), pooled.fields(rp)
        got, err = apply_pooled(pool, fp, bs, nb)
        assert err == 0
        if "lib" in HOST:
            got_k, err_k = apply_pooled_kernel_code(pool_k, rp, bs, nb)
            assert err_k == 0
            np.testing.assert_array_equal(got_k, got)
        ctx = fc["start"].astype(np.int64) + fc["qlen"]
        for s in range(fc["S"]):
            used = -(-int(ctx[s]) // bs)
            np.testing.assert_array_equal(got[s, :used], fc["tables"][s, :used])
    assert next_id > rows  # more sequences than pool rows over the run: rows were reused
