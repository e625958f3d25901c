"""GPU: the whole forward pass and engine against the reference.

  * replayed ModelRunner.execute calls: logits within 1e-3 relative of the
    reference's (measured error is ~1e-6) and the same
    argmax on every row;
  * whole-engine greedy token streams identical to the reference's at every
    block size, chunk budget, batch composition, with preemption, prefix
    caching and speculative decoding (k = 1, 2, 4, 8), on the small test
    model and on the benchmark workloads.
"""

import numpy as np
import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite

pytestmark = [pytest.mark.gpu, needs_vllmlite]

torch = pytest.importorskip("torch")


def model_cfg(shape, **kw):
    from vllmlite.config import ModelConfig

    d = dict(shape)
    d.update(kw)
    return ModelConfig(vocab_size=261, **d)


def engine_cfg(shape, bs=16, nb=512, max_seqs=8, budget=1024, prefix=False, chunked=True, maxlen=None):
    from vllmlite.config import CacheConfig, EngineConfig, SchedulerConfig

    mc = model_cfg(shape)
    if maxlen:
        mc.max_seq_len = maxlen
    return EngineConfig(model=mc,
                        cache=CacheConfig(block_size=bs, num_blocks=nb, enable_prefix_caching=prefix),
                        scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget,
                                                  chunked_prefill=chunked))


def run_prompts(eng, prompts, max_tokens):
    from vllmlite.sequence import SamplingParams

    p = SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True)
    ids = [eng.add_request(x, p) for x in prompts]
    while eng.has_work:
        eng.step()
    return [eng.seqs[i].output_token_ids for i in ids]


def run_requests(eng, reqs):
    ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
    while eng.has_work:
        eng.step()
    return [eng.seqs[i].output_token_ids for i in ids]


@pytest.mark.parametrize("name,bs", [("replay_bench.npz", 16), ("replay_spec.npz", 4)])
def test_runner_replay_logits(name, bs):
    from vllmlite.config import CacheConfig

    from vllt.runner import CudaRunner

    run = CudaRunner(model_cfg(F.BENCH), CacheConfig(block_size=bs, num_blocks=512))
    worst = 0.0
    for seqs, cow, want in F.replay_steps(name):
        got, rows = run.execute(F.as_scheduler_output(seqs, cow))
        assert got.shape == want.shape and got.dtype == np.float32
        rel = np.abs(got - want).max() / np.abs(want).max()
        worst = max(worst, rel)
        assert rel < 1e-3
        assert (got.argmax(1) == want.argmax(1)).all()
    assert worst < 1e-4, worst


@pytest.mark.parametrize("name,bs", [("replay_bench.npz", 16), ("replay_spec.npz", 4)])
def test_device_resident_tables_match_uploaded_tables(name, bs):
    """The runner with its block tables in the device pool (pooled records,
    the default) and with the whole tables uploaded every pass give
    bit-identical logits on the reference's replays."""
    from vllmlite.config import CacheConfig

    from vllt.runner import CudaRunner

    a = CudaRunner(model_cfg(F.BENCH), CacheConfig(block_size=bs, num_blocks=512))
    b = CudaRunner(model_cfg(F.BENCH), CacheConfig(block_size=bs, num_blocks=512), pooled_tables=False)
    for seqs, cow, _ in F.replay_steps(name):
        out = F.as_scheduler_output(seqs, cow)
        for item, s in zip(out.scheduled, seqs):
            item.seq.request_id = f"b{s['block_ids'][0]}"
        la, _ = a.execute(out)
        lb, _ = b.execute(out)
        np.testing.assert_array_equal(la, lb)
    assert a.h2d_bytes < b.h2d_bytes


def test_graph_replay_matches_eager():
    """CUDA-graph replays equal eager runs with the same (bucketed) bounds bit
    for bit; against eager runs with exact bounds they differ only by fp32
    reassociation (the split-K slicing follows the row capacity)."""
    from vllmlite.config import CacheConfig

    from vllt.runner import CudaRunner

    steps = F.replay_steps("replay_spec.npz")
    mk = lambda **kw: CudaRunner(model_cfg(F.BENCH), CacheConfig(block_size=4, num_blocks=512), **kw)
    eager = mk(use_graphs=False)
    eager_b = mk(use_graphs=False, bucket_bounds=True)
    graph = mk(use_graphs=True)
    for seqs, cow, want in steps + steps:  # the second pass replays captured graphs
        out = F.as_scheduler_output(seqs, cow)
        a, _ = eager.execute(out)
        ab, _ = eager_b.execute(out)
        b, _ = graph.execute(out)
        np.testing.assert_array_equal(ab, b)
        np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)
        assert (a.argmax(1) == b.argmax(1)).all()
    assert len(graph.graphs) >= 2 and graph.replayed_kernels > 0


def test_runner_copy_on_write_before_writes():
    """A CoW pair in the same step as the write into the copy (runner.py:63-64)."""
    from vllmlite.config import CacheConfig

    from oracle import model as OM
    from oracle import runner as OR
    from vllt.runner import CudaRunner

    cfg = OM.Shape(vocab_size=261, **F.TINY)
    w = OM.seeded_weights(cfg)
    ref = OR.OracleRunner(cfg, w, 32, 4)
    run = CudaRunner(model_cfg(F.TINY), CacheConfig(block_size=4, num_blocks=32))
    s1 = [dict(start=0, n=6, count=1, tokens=[256, 5, 6, 7, 8, 9], block_ids=[3, 7], drafts=[])]
    # the second sequence shares block 3 fully and the half-filled block 7 is
    # forked into block 11 before its writes
    s2 = [dict(start=6, n=1, count=1, tokens=[10], block_ids=[3, 11], drafts=[]),
          dict(start=6, n=2, count=2, tokens=[12, 13], block_ids=[3, 7], drafts=[14])]
    for seqs, cow in ((s1, []), (s2, [(7, 11)])):
        want, _ = ref.execute(seqs, cow)
        got, _ = run.execute(F.as_scheduler_output(seqs, cow))
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5)


def tiny_reference():
    return F.streams("streams_tiny.npz", "prompts_")


@pytest.mark.parametrize("bs", [1, 4, 16, 64])
def test_block_size_does_not_change_output(bs):
    from vllt.engine import cuda_engine

    assert run_prompts(cuda_engine(engine_cfg(F.TINY, bs=bs)), F.PROMPTS, 20) == tiny_reference()


@pytest.mark.parametrize("budget", [8, 33, 64, 4096])
def test_chunked_prefill_does_not_change_output(budget):
    from vllt.engine import cuda_engine

    assert run_prompts(cuda_engine(engine_cfg(F.TINY, budget=budget)), F.PROMPTS, 20) == tiny_reference()


@pytest.mark.parametrize("max_seqs", [1, 2, 3, 8])
def test_batch_composition_does_not_change_output(max_seqs):
    from vllt.engine import cuda_engine

    assert run_prompts(cuda_engine(engine_cfg(F.TINY, max_seqs=max_seqs)), F.PROMPTS, 20) == tiny_reference()


def test_no_chunking_and_prefix_cache_match():
    from vllt.engine import cuda_engine

    assert run_prompts(cuda_engine(engine_cfg(F.TINY, chunked=False, budget=4096)), F.PROMPTS, 20) == tiny_reference()
    assert run_prompts(cuda_engine(engine_cfg(F.TINY, prefix=True)), F.PROMPTS, 20) == tiny_reference()


@pytest.mark.parametrize("prefix", [False, True])
def test_preemption_preserves_output(prefix):
    from vllt.engine import cuda_engine

    eng = cuda_engine(engine_cfg(F.TINY, bs=4, nb=24, prefix=prefix))
    got = run_prompts(eng, F.PROMPTS, 20)
    assert eng.scheduler.total_preemptions > 0
    assert got == tiny_reference()


@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_speculation_does_not_change_output(k):
    from vllt.engine import cuda_engine, gpu_engine

    assert run_prompts(cuda_engine(engine_cfg(F.TINY), speculative_tokens=k), F.PROMPTS, 20) == tiny_reference()
    eng = gpu_engine(engine_cfg(F.TINY), speculative_tokens=k)
    assert run_prompts(eng, F.REPEATS, 40) == F.streams("streams_tiny.npz", "repeats_")
    assert eng.spec.accepted > 0


def test_gpu_engine_matches_on_prompts_and_frees_blocks():
    from vllt.engine import gpu_engine

    eng = gpu_engine(engine_cfg(F.TINY, bs=4, nb=24, prefix=True))
    assert run_prompts(eng, F.PROMPTS, 20) == tiny_reference()
    a = eng.scheduler.blocks.allocator
    assert eng.scheduler.total_preemptions > 0
    # every block is back: free, or cached with no reference (evictable)
    assert a.num_free == a.num_blocks


def test_bench_workload_mixed_lengths_token_identical():
    """The 48-request mixed-length benchmark: every greedy token equal, with
    the drop-in runner and with device picks (which run ahead: the next
    pass's tokens are resolved on the device from the pick buffer)."""
    from vllt.engine import cuda_engine, gpu_engine
    from vllt.workloads import mixed_workload

    want = F.streams("streams_mixed.npz")
    for make in (cuda_engine, gpu_engine):
        eng = make(engine_cfg(F.BENCH, nb=512, max_seqs=16, budget=1024))
        got = run_requests(eng, mixed_workload(48, 0, 0))
        assert got == want
        assert eng.total_steps == int(F.load("streams_mixed.npz")["steps"])
        if make is gpu_engine:  # greedy ignore_eos: passes launch before the previous tokens are read
            assert eng.passes_ahead >= eng.total_steps // 2


def test_bench_workload_shared_prefix_token_identical():
    from vllt.engine import gpu_engine
    from vllt.workloads import mixed_workload

    eng = gpu_engine(engine_cfg(F.BENCH, nb=768, max_seqs=16, budget=1024, prefix=True, maxlen=768))
    assert run_requests(eng, mixed_workload(48, 0, 256)) == F.streams("streams_shared.npz")
    assert eng.scheduler.blocks.stats()["prefix_hit_rate"] > 0.5


def test_shared_prefix_benchmark_with_device_prefix_hashes():
    """The shared-prefix benchmark with the prefix cache's block hashes
    computed on the device: the reference's token streams, prefix-cache hits,
    and every hash the BlockManager asked for planned ahead."""
    from vllt.engine import gpu_engine
    from vllt.workloads import mixed_workload

    eng = gpu_engine(engine_cfg(F.BENCH, nb=768, max_seqs=16, budget=1024, prefix=True, maxlen=768),
                     device_prefix_hash=True)
    assert run_requests(eng, mixed_workload(48, 0, 256)) == F.streams("streams_shared.npz")
    assert eng.scheduler.blocks.stats()["prefix_hit_rate"] > 0.5
    h = eng.prefix_hasher
    assert h.lookups > 0 and h.misses == 0


@pytest.mark.parametrize("k", [2, 4, 8])
def test_periodic_speculative_token_identical(k):
    from vllt.engine import gpu_engine
    from vllt.workloads import periodic_workload

    eng = gpu_engine(engine_cfg(F.BENCH, nb=4096, max_seqs=64, budget=2048, maxlen=1024), speculative_tokens=k)
    assert run_requests(eng, periodic_workload(128, 0)) == F.streams("streams_periodic.npz")
    assert eng.spec.accepted > 0


def sampled_requests():
    """Seeded temperature requests that exercise every row rule of
    sampling.py:41-64 (min_tokens EOS mask with eos not ignored, repetition
    penalty, top-k, top-p), with prompts longer than the token budget of the
    engines below so that chunked prefill hands the sampler non-final chunks."""
    from vllmlite.sequence import SamplingParams
    from vllmlite.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    out = []
    for i, text in enumerate(F.PROMPTS + F.REPEATS):
        p = SamplingParams(max_tokens=24, temperature=(0.6, 1.0, 1.4)[i % 3], top_k=(0, 20, 5)[i % 3],
                           top_p=(1.0, 0.9, 0.5, 0.95)[i % 4], min_tokens=(0, 6)[i % 2],
                           repetition_penalty=(1.0, 1.3, 0.9)[i % 3], seed=100 + i)
        out.append((f"s{i}", tok.encode(text * 2), p))
    return out


@pytest.mark.parametrize("budget", [16, 1024])
def test_device_sampling_matches_host_sampler(budget):
    """Every token pick on the device (GpuLLMEngine: EOS mask, repetition
    penalty, temperature, top-k, top-p and the draw, no host sampler) equals
    the reference's own sample() run on the host over the same CudaRunner
    logits (cuda_engine: an unmodified LLMEngine), request by request with the
    same seeds. A 16-token budget chunks every prompt: the request's generator
    must not advance on chunks that leave tokens uncomputed."""
    from vllt.engine import cuda_engine, gpu_engine

    reqs = sampled_requests()
    want = run_requests(cuda_engine(engine_cfg(F.TINY, budget=budget)), reqs)
    eng = gpu_engine(engine_cfg(F.TINY, budget=budget))
    got = run_requests(eng, reqs)
    assert got == want
    assert sum(len(t) for t in got) > 100


def test_device_sampling_matches_reference_engine_when_chunked():
    """A seeded temperature request whose prompt exceeds the token budget,
    through GpuLLMEngine and through the reference NumPy engine: the same
    tokens (the fp32 logits agree to ~1e-6, far inside the sampler's margins
    for this seed)."""
    from vllmlite.engine import LLMEngine

    from vllt.engine import gpu_engine

    reqs = sampled_requests()[:3]
    want = run_requests(LLMEngine(engine_cfg(F.TINY, budget=16)), reqs)
    assert run_requests(gpu_engine(engine_cfg(F.TINY, budget=16)), reqs) == want
