"""CPU: GpuLLMEngine's host logic against the reference engine, token for token.

GpuLLMEngine moves every token pick to the device. Its host half decides
which rows are masked, penalised or sampled, builds the seen-token bitmaps,
draws each request's uniform from its own generator (only on the pass that
completes the sequence) and maps picks back to sequences. That half runs here
on the CPU, unchanged, with two test stand-ins:
  * the runner returns the reference NumpyRunner's own logits for each pass;
  * the library's sampling entry points are carried out by the oracle
    (oracle/sampling.py, pinned to the reference's sample() by
    tests/test_oracle_golden.py) on the same host buffers, reached through the
    pointers the engine passes, exactly as the C ABI receives them.
So any difference from the reference LLMEngine comes from the engine's own
bookkeeping. The tensor-parallel branch (vocab-parallel argmax, full rows
gathered for masked / penalised / sampled rows) runs the same way with a
runner that reports two shards.
"""

import ctypes
from types import SimpleNamespace as NS

import numpy as np
import pytest

from oracle import sampling as SP
from tests import fixtures as F
from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite


def view(ptr, dtype, n):
    """numpy view of n elements at a host address (None for NULL)."""
    if not ptr:
        return None
    ct = np.ctypeslib.as_ctypes_type(np.dtype(dtype))
    return np.ctypeslib.as_array((ct * n).from_address(ptr))


def seen_of(bits, r, words):
    if bits is None:
        return []
    row = bits[r * words:(r + 1) * words]
    return [c for c in range(words * 32) if (int(row[c >> 5]) >> (c & 31)) & 1]


class OracleLib:
    """The three sampling entry points of include/vllt.h, computed by the oracle."""

    def __init__(self):
        self.calls = {"greedy": 0, "top_p": 0, "accept": 0}

    def vllt_sample_greedy(self, logits, rows, vocab, ld, mask, eos, pen, bits, out, stream):
        self.calls["greedy"] += 1
        x = view(logits, np.float32, rows * ld).reshape(rows, ld)
        m, p = view(mask, np.uint8, rows), view(pen, np.float32, rows)
        o = view(out, np.int32, rows)
        words = (vocab + 31) // 32
        b = view(bits, np.uint32, rows * words)
        for r in range(rows):
            masked = m is not None and m[r]
            o[r] = SP.greedy(x[r, :vocab], eos_id=eos if masked else None, num_generated=0,
                             min_tokens=1 if masked else 0, seen=seen_of(b, r, words),
                             penalty=float(p[r]) if p is not None else 1.0)
        return 0

    def vllt_sample_top_p(self, logits, rows, vocab, ld, n_logit_rows, row_index, mask, eos, pen, bits, temp,
                          top_k, top_p, u, out, stream):
        self.calls["top_p"] += 1
        x = view(logits, np.float32, n_logit_rows * ld).reshape(n_logit_rows, ld)
        ri = view(row_index, np.int32, rows)
        m, p = view(mask, np.uint8, rows), view(pen, np.float32, rows)
        t, k, tp = view(temp, np.float32, rows), view(top_k, np.int32, rows), view(top_p, np.float32, rows)
        uu, o = view(u, np.float64, rows), view(out, np.int32, rows)
        words = (vocab + 31) // 32
        b = view(bits, np.uint32, rows * words)
        for r in range(rows):
            src = int(ri[r]) if ri is not None else r
            if not 0 <= src < n_logit_rows:  # the kernel's answer to a row outside the buffer
                o[r] = -1
                continue
            masked = m is not None and m[r]
            o[r], _, _ = SP.sample_with_uniform(
                x[src, :vocab], float(t[r]), int(k[r]), float(tp[r]), float(uu[r]),
                eos_id=eos if masked else None, num_generated=0, min_tokens=1 if masked else 0,
                seen=seen_of(b, r, words), penalty=float(p[r]) if p is not None else 1.0)
        return 0

    def vllt_spec_accept(self, cu, drafts, doff, S, picks, acc, stream):
        self.calls["accept"] += 1
        c, o = view(cu, np.int32, S + 1), view(doff, np.int32, S)
        nd = int(c[S] - c[0])
        d = view(drafts, np.int32, max(nd, 1))
        pk, a = view(picks, np.int32, int(c[S])), view(acc, np.int32, S)
        for s in range(S):
            n, j = int(c[s + 1] - c[s] - 1), 0
            while j < n and pk[c[s] + j] == d[o[s] + j]:
                j += 1
            a[s] = j
        return 0


class ReferenceLogitsRunner:
    """Stands in for CudaRunner: each pass's logits are the reference
    NumpyRunner's, left in a host buffer laid out like logits_dev
    ([rows][vocab_padded] fp32)."""

    tp_size = 1

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, device=None, lib=None):
        from vllmlite.runner import NumpyRunner

        from vllt.runner import CudaRunner

        self.check_step_flags = CudaRunner.check_step_flags.__get__(self)
        self.meta = torch.zeros(16, dtype=torch.int32)  # word 7: the metadata builder's error flags
        self.packer = object()
        self.ref = NumpyRunner(model_cfg, cache_cfg)
        self.model_cfg = model_cfg
        self.dev = torch.device("cpu")
        self.L = lib
        self.w = NS(vocab_padded=(model_cfg.vocab_size + 3) // 4 * 4)
        self.passes = 0

    def launch(self, out):
        logits, rows = self.ref.execute(out)
        R = logits.shape[0]
        self.logits_dev = torch.zeros((max(R, 1), self.w.vocab_padded), dtype=torch.float32)
        self.logits_dev[:R, :logits.shape[1]] = torch.from_numpy(logits)
        self.passes += 1
        return rows, R


class TwoShardRunner(ReferenceLogitsRunner):
    """The tensor-parallel runner's interface with two vocabulary shards: the
    vocab-parallel argmax and the gather of full rows."""

    tp_size = 2

    def greedy_picks(self, R):
        V = self.model_cfg.vocab_size
        return torch.from_numpy(self.logits_dev[:R, :V].numpy().argmax(1).astype(np.int32))

    def gather_rows(self, rows):
        V = self.model_cfg.vocab_size
        self.gathered = getattr(self, "gathered", 0) + len(rows)
        return self.logits_dev[torch.as_tensor(rows, dtype=torch.int64), :V].contiguous()


def engine_cfg(budget, max_seqs=8, bs=16, nb=512):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    return EngineConfig(model=ModelConfig(vocab_size=261, **F.TINY),
                        cache=CacheConfig(block_size=bs, num_blocks=nb),
                        scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget))


def requests():
    """Seeded requests covering every row rule of sampling.py:41-64: greedy,
    greedy with min_tokens (EOS not ignored) and a repetition penalty,
    temperature with top-k / top-p / penalty / min_tokens; prompts longer than
    a 16-token budget so chunked prefill produces non-final chunks."""
    from vllmlite.sequence import SamplingParams
    from vllmlite.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    out = []
    for i, text in enumerate(F.PROMPTS + F.REPEATS):
        if i % 4 == 3:
            p = SamplingParams(max_tokens=12, temperature=0.0, min_tokens=4, repetition_penalty=1.4)
        else:
            p = SamplingParams(max_tokens=12, temperature=(0.6, 1.0, 1.4)[i % 3], top_k=(0, 20, 5)[i % 3],
                               top_p=(1.0, 0.9, 0.5, 0.95)[i % 4], min_tokens=(0, 6)[i % 2],
                               repetition_penalty=(1.0, 1.3, 0.9)[i % 3], seed=100 + i)
        out.append((f"s{i}", tok.encode(text * 2), p))
    return out


def run(eng, reqs):
    ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
    while eng.has_work:
        eng.step()
    return [eng.seqs[i].output_token_ids for i in ids]


def gpu_engine_on_host(runner_cls, cfg, k=0):
    import vllt._lib as _lib
    from vllt.engine import GpuLLMEngine, cuda_engine

    lib = OracleLib()
    eng = cuda_engine(cfg, speculative_tokens=k, engine_cls=GpuLLMEngine.resolve(), runner_cls=runner_cls,
                      lib=lib)
    return eng, lib


@pytest.fixture(autouse=True)
def _no_stream(monkeypatch):
    import vllt._lib as _lib

    monkeypatch.setattr(_lib, "stream_handle", lambda stream=None: 0)


@pytest.mark.parametrize("runner_cls", [ReferenceLogitsRunner, TwoShardRunner])
@pytest.mark.parametrize("budget", [16, 1024])
def test_device_pick_plumbing_matches_reference_engine(runner_cls, budget):
    from vllmlite.engine import LLMEngine

    reqs = requests()
    want = run(LLMEngine(engine_cfg(budget)), reqs)
    eng, lib = gpu_engine_on_host(runner_cls, engine_cfg(budget))
    got = run(eng, reqs)
    assert got == want
    assert lib.calls["top_p"] > 0
    if runner_cls is TwoShardRunner:
        assert eng.runner.gathered > 0 and lib.calls["greedy"] > 0
    # a 16-token budget chunks every prompt: passes outnumber those of the 1024 budget
    assert eng.runner.passes > len(reqs)


def test_speculative_picks_match_reference_engine():
    """Verify rows take plain argmax and the accept rule; the n-gram proposer
    and commit are the reference's own."""
    from vllmlite.engine import LLMEngine
    from vllmlite.sequence import SamplingParams
    from vllmlite.tokenizer import ByteTokenizer

    tok = ByteTokenizer()
    p = SamplingParams(max_tokens=30, temperature=0.0, ignore_eos=True)
    reqs = [(f"r{i}", tok.encode(t), p) for i, t in enumerate(F.REPEATS)]
    want = run(LLMEngine(engine_cfg(1024), speculative_tokens=4), reqs)
    eng, lib = gpu_engine_on_host(ReferenceLogitsRunner, engine_cfg(1024), k=4)
    assert run(eng, reqs) == want
    assert lib.calls["accept"] > 0 and eng.spec.accepted > 0


def test_generator_advances_only_on_completing_passes():
    """A seeded temperature request with a 40-token prompt under a 16-token
    budget: the first two passes leave tokens uncomputed and must not draw."""
    from vllmlite.sequence import SamplingParams

    from vllt.engine import completes, pick_inputs

    seq = NS(num_tokens=40, draft_token_ids=[], output_token_ids=[],
             params=SamplingParams(temperature=1.0, seed=3), request_id="a")
    for start, n, final in ((0, 16, False), (16, 16, False), (32, 8, True)):
        item = NS(seq=seq, start_pos=start, num_tokens=n)
        assert completes(item) == final
        sampled = pick_inputs([item], [(0, 1)], 1, 257)[5]
        assert sampled == ([(0, 0)] if final else [])


def test_a_pass_the_device_flagged_raises_and_reloads_the_tables():
    """The metadata builder's error word comes back with the picks: a flagged
    pass raises instead of committing tokens, and the runner drops its
    packer so the next pass uploads whole tables."""
    from vllmlite.sequence import SamplingParams

    eng, lib = gpu_engine_on_host(ReferenceLogitsRunner, engine_cfg(1024))
    eng.add_request(params=SamplingParams(max_tokens=4, temperature=0.0), request_id="x",
                    prompt_token_ids=[256, 1, 2, 3])
    eng.runner.meta[7] = 2
    with pytest.raises(RuntimeError, match="flags 2"):
        eng.step()
    assert eng.runner.packer is None
    assert eng.seqs["x"].output_token_ids == []


@pytest.mark.parametrize("workload", ["mixed", "shared"])
def test_benchmark_streams_through_the_device_pick_path(workload, tmp_path):
    """The reference's 48-request benchmarks (C1; C2 with the prefix cache,
    its block hashes planned and computed by the device hash code compiled
    for the host) through GpuLLMEngine's host path: every greedy token and
    the number of engine steps equal the reference run's golden streams."""
    import ctypes

    from tests.host_build import build_harness
    from tests.test_prefix_hash import chain_host
    from vllt.engine import GpuLLMEngine, cuda_engine
    from vllt.prefix_hash import DevicePrefixHasher
    from vllt.workloads import mixed_workload

    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    shared = workload == "shared"
    host = build_harness("prefix_hash_host", str(tmp_path)) if shared else None
    if shared and host is None:
        pytest.skip("g++ is not available")

    class Lib(OracleLib):
        def vllt_prefix_hash_chains(self, tokens, tok_off, nblk, out_off, prev, n, bs, out, stream):
            nb = view(nblk, np.int32, n)
            to, oo = view(tok_off, np.int64, n), view(out_off, np.int64, n)
            o = view(out, np.uint8, 32 * max(int(oo[-1] + nb[-1]) if n else 0, 1))
            for c in range(n):
                toks = view(tokens + 4 * int(to[c]), np.int32, max(int(nb[c]) * bs, 1))[:int(nb[c]) * bs]
                p = bytes(view(prev + 32 * c, np.uint8, 32)) if prev else b"\0"
                for b, h in enumerate(chain_host(host, p.decode() if p[0] else None, toks, bs)):
                    o[32 * (int(oo[c]) + b):32 * (int(oo[c]) + b + 1)] = np.frombuffer(h.encode(), np.uint8)
            return 0

    if shared:
        host.hash_chain_host.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 2 + [ctypes.c_void_p]
    maxlen = 768 if shared else 512
    cfg = EngineConfig(model=ModelConfig(vocab_size=261, **dict(F.BENCH, max_seq_len=maxlen)),
                       cache=CacheConfig(block_size=16, num_blocks=maxlen, enable_prefix_caching=shared),
                       scheduler=SchedulerConfig(max_seqs=16, max_batched_tokens=1024))
    lib = Lib()
    eng = cuda_engine(cfg, engine_cls=GpuLLMEngine.resolve(), runner_cls=ReferenceLogitsRunner, lib=lib)
    if shared:
        eng.prefix_hasher = DevicePrefixHasher(eng, lib=lib)
    got = run(eng, mixed_workload(48, 0, 256 if shared else 0))
    assert got == F.streams(f"streams_{workload}.npz")
    assert eng.total_steps == int(F.load(f"streams_{workload}.npz")["steps"])
    if shared:
        assert eng.prefix_hasher.misses == 0 and eng.prefix_hasher.lookups > 0
