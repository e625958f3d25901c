"""CPU: the whole device path of GpuLLMEngine, its own compiled code, against
the reference engine's token streams.

HostRunner gives GpuLLMEngine libvllt's fp32 path built for the host
(tests/host_build.py build_library_host). It keeps CudaRunner's state in
host memory and uses the runner's own pieces: packer, descriptor, bucketed
bounds, pick buffer and error check. So every pass goes through the same
code as on the GPU:
  * the engine's scheduling and bookkeeping, including run-ahead;
  * the pooled step record with stand-in tokens;
  * vllt_forward with the compiled metadata builder (which resolves the
    stand-ins), RMSNorm, SGEMM epilogues and attention;
  * vllt_sample_greedy's compiled kernel, the pick buffer and the error word.

The benchmarks' requests must give the token streams the reference engine
gave (tests/golden/streams_*.npz): C1 (mixed lengths), C2 (a 256-token shared
prefix with the prefix cache, so copy-on-write runs through the compiled
copy kernel) and C5 (periodic prompts with speculative k = 4, verified by
the compiled accept kernel against the k = 0 streams). Greedy streams do not
depend on which requests share a batch, so a subset of each is run.

The C4 serving path (HostLlamaRunner: LlamaRunner's bf16 weights, caches and
descriptor) runs the same way on a narrow Llama-shaped model, against the
reference's LLMEngine over the same runner.
"""

import pytest

from tests import fixtures as F
from tests.conftest import needs_vllmlite
from tests.host_runner import HostRunner

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite


@pytest.fixture
def host_lib(host_library):
    return host_library


@pytest.fixture(autouse=True)
def _no_stream(monkeypatch):
    import vllt._lib as _lib

    monkeypatch.setattr(_lib, "stream_handle", lambda stream=None: 0)


def fixture_streams(name):
    z = F.load(name)
    out, o = [], 0
    for n in z["lens"]:
        out.append(z["tokens"][o:o + int(n)].tolist())
        o += int(n)
    return out


@pytest.mark.parametrize("workload,pick,maxlen,nb,prefix,spec,seqs,budget", [
    ("mixed", [1, 9, 30, 46], 512, 512, False, 0, 16, 1024),           # C1, run-ahead
    ("shared", [0, 7, 15, 33], 768, 768, True, 0, 16, 384),            # C2: prefix cache hits, run-ahead
    ("periodic", [0, 5], 1024, 4096, False, 4, 64, 2048),             # C5: speculative k = 4
])
def test_engine_streams_through_the_compiled_device_path(host_lib, workload, pick, maxlen, nb, prefix, spec, seqs,
                                                          budget):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    from vllt.engine import GpuLLMEngine, cuda_engine
    from vllt.workloads import mixed_workload, periodic_workload

    if workload == "periodic":
        reqs, want_all = periodic_workload(128, seed=0), fixture_streams("streams_periodic.npz")
    else:
        reqs = mixed_workload(48, 0, 256 if workload == "shared" else 0)
        want_all = fixture_streams(f"streams_{workload}.npz")
    HostRunner.lib = host_lib
    shape = {k: v for k, v in F.BENCH.items() if k != "max_seq_len"}
    cfg = EngineConfig(model=ModelConfig(vocab_size=261, max_seq_len=maxlen, **shape),
                       cache=CacheConfig(block_size=16, num_blocks=nb, enable_prefix_caching=prefix),
                       scheduler=SchedulerConfig(max_seqs=seqs, max_batched_tokens=budget))
    eng = cuda_engine(cfg, speculative_tokens=spec, engine_cls=GpuLLMEngine.resolve(), runner_cls=HostRunner)
    ids = [eng.add_request(params=reqs[i][2], request_id=reqs[i][0], prompt_token_ids=reqs[i][1]) for i in pick]
    while eng.has_work:
        eng.step()
    got = [eng.seqs[i].output_token_ids for i in ids]
    assert got == [want_all[i] for i in pick]
    if spec:  # proposals read the new tokens: no pass runs ahead; drafts were verified on the device
        assert eng.passes_ahead == 0 and eng.spec.accepted > 0
    else:
        assert eng.passes_ahead >= eng.total_steps // 2 and eng.runner.stand_ins > 0
    if prefix:
        assert eng.scheduler.blocks.allocator.hits > 0


def test_llama_engine_through_the_compiled_bf16_path(host_lib):
    """The C4 serving path (the bench's gpu_engine with LlamaRunner) on a
    narrow Llama-shaped model: GpuLLMEngine over the bf16 host runner (device
    greedy and temperature picks, run-ahead) gives the token streams of the
    reference's unmodified LLMEngine over the same runner, whose host
    sample() reads the logits the same compiled forward produced. Chunked
    prefill (budget 96) and a prompt past 256 tokens put tensor-core prefill
    tiles over cached prefixes in the passes; decode rows take the TMA decode
    kernel and every projection a tcgen05 GEMM."""
    import numpy as np
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig
    from vllmlite.sequence import SamplingParams

    from tests.host_runner import HostLlamaRunner
    from vllt.engine import GpuLLMEngine, cuda_engine

    HostLlamaRunner.lib = host_lib
    host_lib.vllt_host_mma_count.restype = __import__("ctypes").c_int64
    mc = ModelConfig(n_layers=2, n_heads=2, n_kv_heads=1, d_model=256, d_ff=512, vocab_size=300, max_seq_len=1024,
                     seed=3)
    cfg = EngineConfig(model=mc, cache=CacheConfig(block_size=16, num_blocks=96),
                       scheduler=SchedulerConfig(max_seqs=4, max_batched_tokens=96))
    rng = np.random.default_rng(5)
    prompts = [[int(t) for t in rng.integers(1, 300, size=n)] for n in (40, 300, 7, 120)]
    params = [SamplingParams(max_tokens=10, temperature=0.0, ignore_eos=True) for _ in range(3)]
    params.append(SamplingParams(max_tokens=10, temperature=0.8, top_p=0.9, seed=11, ignore_eos=True))

    def streams(eng):
        ids = [eng.add_request(params=p, prompt_token_ids=t) for t, p in zip(prompts, params)]
        while eng.has_work:
            eng.step()
        return [eng.seqs[i].output_token_ids for i in ids]

    mma0 = host_lib.vllt_host_mma_count()
    want = streams(cuda_engine(cfg, runner_cls=HostLlamaRunner))
    eng = cuda_engine(cfg, engine_cls=GpuLLMEngine.resolve(), runner_cls=HostLlamaRunner)
    assert streams(eng) == want
    assert all(len(s) == 10 for s in want)
    assert eng.passes_ahead > 0
    assert host_lib.vllt_host_mma_count() > mma0


@pytest.mark.parametrize("tp_size", [1, 2])
def test_copy_on_write_copies_the_runners_own_cache_layout(host_lib, tp_size):
    """CudaRunner.copy_blocks_on_device (the copy-on-write of a forked block,
    runner.py:54-60) on the bf16 Llama runner's caches: the element type and
    the KV heads of this rank come from the caches themselves (a rank under
    tensor parallelism holds n_kv / tp_size heads), every layer copied, no
    other block touched."""
    import numpy as np
    from vllmlite.config import CacheConfig, ModelConfig

    from tests.host_runner import HostLlamaRunner

    class Shard(HostLlamaRunner):
        pass

    Shard.lib, Shard.tp_size, Shard.tp_rank, Shard.tp_comm = host_lib, tp_size, tp_size - 1, 0x7C
    from types import SimpleNamespace

    mc = ModelConfig(n_layers=2, n_heads=4, n_kv_heads=2, d_model=512, d_ff=512, vocab_size=300, max_seq_len=256,
                     seed=3)
    run = Shard(mc, CacheConfig(block_size=16, num_blocks=12), SimpleNamespace(max_seqs=2, max_batched_tokens=32))
    assert run.cache_k.shape == (2, 12, 2 // tp_size, 16, 128) and run.cache_k.dtype == torch.bfloat16
    g = torch.Generator().manual_seed(tp_size)
    run.cache_k.copy_(torch.randn(run.cache_k.shape, generator=g).to(torch.bfloat16))
    run.cache_v.copy_(torch.randn(run.cache_v.shape, generator=g).to(torch.bfloat16))
    want_k, want_v = run.cache_k.clone(), run.cache_v.clone()
    pairs = np.asarray([[3, 7], [0, 11]], np.int32)
    for s, d in pairs:
        want_k[:, d], want_v[:, d] = want_k[:, s], want_v[:, s]
    run.copy_blocks_on_device(pairs.ctypes.data, len(pairs))
    assert torch.equal(run.cache_k, want_k) and torch.equal(run.cache_v, want_v)
