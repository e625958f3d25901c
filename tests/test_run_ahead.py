"""CPU: the engine's run-ahead against the reference engine.

GpuLLMEngine schedules and launches pass N+1 before pass N's tokens reach the
host when no sequence completing pass N can stop on a token's value
(stops_on_length). Each new token is then a stand-in id -1 - j (j: its entry
in the device pick buffer) until the engine writes the picked token over it.
The next pass's packed record carries the stand-ins, and the device
metadata builder resolves them (resolve_token in csrc/meta_items.cuh).

Here the runner packs every pass with the real StepPacker (pooled tables),
builds the metadata with the builder's code compiled for the host
(tests/meta_host.cpp) using its pick buffer as the token source, and checks
that the resolved tokens are the true ones. Logits come from the reference
NumpyRunner, and picks from the oracle through the C-ABI pick entry points.
Against the reference LLMEngine (vllmlite/engine.py:99-181), call by call:
  * every step() returns the same outputs (request, new tokens, finished,
    reason), the token streams and the step count are equal, and the prefix
    cache's hits and misses are equal;
  * with greedy ignore_eos requests (the benchmark's) nearly every pass runs
    ahead. With requests that can stop on EOS, or with seeded sampling, only
    the passes whose completing sequences stop on length do;
  * a cache small enough to preempt (recompute prompts end in stand-ins)
    gives the same result, and the allocator ends where the reference's does.
"""

import ctypes

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite
from tests.test_engine_host import OracleLib, ReferenceLogitsRunner

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite


@pytest.fixture(scope="module")
def meta_host(tmp_path_factory):
    from tests.host_build import build_harness

    lib = build_harness("meta_host", str(tmp_path_factory.mktemp("meta_ahead")))
    if lib is None:
        pytest.skip("g++ is not available")
    lib.build_meta_host.argtypes = ([ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 8 +
                                    [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int])
    return lib


@pytest.fixture(autouse=True)
def _no_stream(monkeypatch):
    import vllt._lib as _lib

    monkeypatch.setattr(_lib, "stream_handle", lambda stream=None: 0)


class AheadRunner(ReferenceLogitsRunner):
    """ReferenceLogitsRunner with CudaRunner's pick buffer and record path."""

    meta_lib = None
    PICK_WORDS = 4096

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, device=None, lib=None):
        from vllt import _lib
        from vllt.runner import StepPacker, tile_positions

        super().__init__(model_cfg, cache_cfg, sched_cfg, device, lib)
        self.picks_dev = torch.zeros(self.PICK_WORDS, dtype=torch.int32)
        self.bs, self.nb = cache_cfg.block_size, cache_cfg.num_blocks
        self.caps = _lib.Caps(64, 4096, 256, -(-model_cfg.max_seq_len // self.bs))
        self.qp = tile_positions(model_cfg.n_heads // model_cfg.n_kv_heads)
        self.packer = StepPacker(self.bs, self.nb, model_cfg.vocab_size, model_cfg.max_seq_len, self.qp,
                                 pool_slots=128, pool_width=self.caps.max_table_width, token_refs=self.PICK_WORDS)
        self.pool = np.full((128, self.caps.max_table_width), -1, np.int32)
        self.stand_ins = 0

    def pick_buffer(self, n):
        return self.picks_dev[:n]

    def launch(self, out):
        from vllt import _lib
        from vllt.runner import _tokens

        rec = self.packer.pack(out)[0]
        self.stand_ins += int((rec[5 + 3 * rec[0]:5 + 3 * rec[0] + rec[1]] < 0).sum())
        L = _lib.lib()
        meta = np.zeros(L.vllt_meta_bytes(ctypes.byref(self.caps)) // 4, np.int32)
        picks = self.picks_dev.numpy()
        rec = np.ascontiguousarray(rec, np.int32)
        err = self.meta_lib.build_meta_host(rec.ctypes.data, self.pool.ctypes.data, self.pool.shape[0],
                                            self.caps.max_seqs, self.caps.max_tokens, self.caps.max_rows,
                                            self.caps.max_table_width, self.bs, self.nb, self.qp,
                                            meta.ctypes.data, picks.ctypes.data, picks.size,
                                            self.model_cfg.vocab_size)
        assert err == 0
        off = (L.vllt_meta_field(ctypes.c_void_p(meta.ctypes.data), ctypes.byref(self.caps), 8)
               - meta.ctypes.data) // 4
        device_tokens = meta[off:off + int(rec[1])].tolist()
        # the true tokens: stand-ins replaced by the picks they refer to
        saved = []
        for item in out.scheduled:
            o = item.seq.output_token_ids
            for k, t in enumerate(o):
                if t < 0:
                    saved.append((o, k, t))
                    o[k] = int(picks[-t - 1])
        try:
            want = [t for item in out.scheduled for t in _tokens(item.seq, item.start_pos, item.num_tokens)]
            assert device_tokens == want
            return super().launch(out)
        finally:
            for o, k, t in saved:  # the engine writes the tokens over its stand-ins itself
                o[k] = t


def make_engine(cfg, meta_host, run_ahead=True):
    from vllt.engine import GpuLLMEngine, cuda_engine

    AheadRunner.meta_lib = meta_host
    eng = cuda_engine(cfg, engine_cls=GpuLLMEngine.resolve(), runner_cls=AheadRunner, lib=OracleLib())
    eng.run_ahead = run_ahead
    return eng


def drive(eng, reqs):
    """Per step() call: [(request, new tokens, finished, reason)], then the streams."""
    ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
    calls = []
    while eng.has_work:
        calls.append([(o.request_id, list(o.new_token_ids), o.finished, o.finish_reason) for o in eng.step()])
    return calls, [eng.seqs[i].output_token_ids for i in ids]


def config(budget=64, max_seqs=8, bs=16, nb=512, prefix=False, max_len=512, chunked=True):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    return EngineConfig(model=ModelConfig(vocab_size=261, **dict(F.TINY, max_seq_len=max_len)),
                        cache=CacheConfig(block_size=bs, num_blocks=nb, enable_prefix_caching=prefix),
                        scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget,
                                                  chunked_prefill=chunked))


def bench_requests(n=12, shared=0, max_tokens=None):
    from vllt.workloads import mixed_workload

    reqs = mixed_workload(n, 3, shared)
    if max_tokens:
        for _, _, p in reqs:
            p.max_tokens = min(p.max_tokens, max_tokens)
    return reqs


def compare(cfg, reqs, meta_host):
    from vllmlite.engine import LLMEngine

    ref = LLMEngine(cfg)
    want_calls, want = drive(ref, reqs)
    eng = make_engine(cfg, meta_host)
    got_calls, got = drive(eng, reqs)
    assert got == want
    assert got_calls == want_calls
    assert eng.total_steps == ref.total_steps and eng.total_output_tokens == ref.total_output_tokens
    a, b = eng.scheduler.blocks.allocator, ref.scheduler.blocks.allocator
    assert (a.hits, a.misses) == (b.hits, b.misses)
    assert a.num_free == b.num_free  # the reference's count (a block whose hash is cached twice is not returned)
    return eng, ref


@pytest.mark.parametrize("budget", [64, 1024])
def test_benchmark_requests_run_ahead_and_match(meta_host, budget):
    eng, ref = compare(config(budget), bench_requests(12, max_tokens=40), meta_host)
    assert eng.passes_ahead >= eng.total_steps - 2 and eng.runner.stand_ins > 0


def test_shared_prefix_with_prefix_cache(meta_host):
    eng, ref = compare(config(128, bs=16, nb=512, prefix=True, max_len=768),
                       bench_requests(10, shared=64, max_tokens=30), meta_host)
    assert ref.scheduler.blocks.allocator.hits > 0 and eng.passes_ahead > 0


def test_preemption_with_stand_ins(meta_host):
    eng, ref = compare(config(96, max_seqs=8, bs=8, nb=40), bench_requests(10, max_tokens=48), meta_host)
    assert ref.scheduler.total_preemptions > 0 and eng.passes_ahead > 0 and eng.runner.stand_ins > 0


def test_mixed_stop_rules_run_ahead_only_where_allowed(meta_host):
    """EOS-stopping greedy rows, seeded temperature rows with top-k / top-p /
    penalties, and ignore_eos rows in one batch: a pass runs ahead only when
    every completing sequence stops on length."""
    from vllmlite.sequence import SamplingParams

    from tests.test_engine_host import requests

    reqs = requests()
    for i, (_, _, p) in enumerate(reqs):
        if i % 3 == 0:
            p.ignore_eos = True
    rid, ids, _ = bench_requests(1)[0]
    reqs.append(("long", ids, SamplingParams(max_tokens=60, temperature=0.0, ignore_eos=True)))
    eng, ref = compare(config(16), reqs, meta_host)
    assert 0 < eng.passes_ahead < eng.total_steps


def test_stops_on_length_rules():
    from vllmlite.sequence import SamplingParams

    from vllt.engine import stops_on_length

    assert stops_on_length(SamplingParams(ignore_eos=True), 2)
    assert stops_on_length(SamplingParams(ignore_eos=True, stop_token_ids=[5]), 2)  # ignore_eos skips them too
    assert not stops_on_length(SamplingParams(), 2)
    assert stops_on_length(SamplingParams(), None)
    assert not stops_on_length(SamplingParams(stop_token_ids=[5]), None)
    assert not stops_on_length(SamplingParams(ignore_eos=True, stop=["x"]), 2)


def test_abort_between_calls_while_a_pass_runs_ahead(meta_host):
    """A request aborted while its next pass is already launched: later
    outputs never mention it, every other stream equals the reference run's
    (batch-invariant picks), and every block comes back."""
    from vllmlite.engine import LLMEngine

    cfg = config(64)
    reqs = bench_requests(8, max_tokens=30)
    ref = LLMEngine(cfg)
    _, want = drive(ref, reqs)
    eng = make_engine(cfg, meta_host)
    ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
    victim, after = ids[2], []
    for _ in range(12):
        eng.step()
    assert eng._next is not None and eng.abort(victim)
    while eng.has_work:
        after += [o for o in eng.step() if o.request_id == victim and o.new_token_ids]
    assert after == []
    got = [eng.seqs[i].output_token_ids for i in ids]
    for i in range(len(ids)):
        if ids[i] != victim:
            assert got[i] == want[i]
    n = len(got[2])
    assert 0 < n < len(want[2]) and got[2] == want[2][:n] and min(got[2]) >= 0
    a, b = eng.scheduler.blocks.allocator, ref.scheduler.blocks.allocator
    assert a.num_free == b.num_free == a.num_blocks


def test_first_token_time_is_taken_when_the_token_is_on_the_host(meta_host):
    eng = make_engine(config(1024), meta_host)
    reqs = bench_requests(4, max_tokens=8)
    ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
    while eng.has_work:
        for o in eng.step():
            seq = eng.seqs[o.request_id]
            assert min(seq.output_token_ids) >= 0  # no stand-in is ever visible in an output
            assert seq.first_token_at is not None and seq.first_token_at >= seq.arrival
    assert eng.passes_ahead > 0 and all(eng.seqs[i].finished_at >= eng.seqs[i].first_token_at for i in ids)


def prompt_requests(max_tokens=20):
    """The fixture prompts, greedy with ignore_eos (the reference's invariance tests' requests)."""
    from vllmlite.sequence import SamplingParams
    from vllmlite.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    return [(f"p{i}", tok.encode(t), SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True))
            for i, t in enumerate(F.PROMPTS)]


# the reference's invariance grid (tests/test_engine.py:57-110), with run-ahead on
@pytest.mark.parametrize("kw", [dict(bs=1), dict(bs=4), dict(bs=64), dict(prefix=True),
                                dict(budget=8), dict(budget=33), dict(budget=4096),
                                dict(budget=4096, chunked=False), dict(max_seqs=1), dict(max_seqs=2),
                                dict(max_seqs=3), dict(bs=4, nb=24), dict(bs=4, nb=24, prefix=True)],
                         ids=lambda kw: ",".join(f"{k}={v}" for k, v in kw.items()))
def test_reference_invariance_grid(meta_host, kw):
    cfg = dict(budget=1024, max_seqs=8, bs=16, nb=512)
    cfg.update(kw)
    eng, ref = compare(config(**cfg), prompt_requests(), meta_host)
    assert eng.passes_ahead > 0
    if cfg["nb"] == 24:
        assert ref.scheduler.total_preemptions > 0
