"""GPU: the bf16 Llama-shaped forward (tcgen05 GEMMs) against an fp32 GPU re-run.

The reference has no bf16 path and no checkpoint at this shape; the bf16 model
is validated against the fp32 parity path (itself pinned to the reference's
NumPy forward) running the SAME weights (the bf16 values, widened to fp32).

Stated tolerance: max |logit_bf16 - logit_fp32| <= 5e-2 * max |logit_fp32| per
step, and the greedy pick agrees on every row whose fp32 top-1 / top-2 gap is
larger than twice that step's measured error (rows closer than that are
near-ties that bf16 rounding of the activations may legitimately flip).
"""

import numpy as np
import pytest

from tests import fixtures as F

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def schedule(vocab, rng):
    """Three passes: mixed chunked prefill and decode, then a verify row set."""
    def toks(n):
        return [int(t) for t in rng.integers(0, vocab, size=n)]

    a, b, c = toks(41), toks(150), toks(1)
    return [
        [dict(start=0, n=41, count=1, tokens=a, block_ids=[0, 1, 2], drafts=[]),
         dict(start=0, n=100, count=1, tokens=b[:100], block_ids=[3, 4, 5, 6, 7, 8, 9], drafts=[]),
         dict(start=0, n=1, count=1, tokens=c, block_ids=[10], drafts=[])],
        [dict(start=41, n=1, count=1, tokens=toks(1), block_ids=[0, 1, 2], drafts=[]),
         dict(start=100, n=50, count=1, tokens=b[100:], block_ids=[3, 4, 5, 6, 7, 8, 9, 11, 12, 13], drafts=[]),
         dict(start=1, n=1, count=1, tokens=toks(1), block_ids=[10], drafts=[])],
        [dict(start=42, n=4, count=4, tokens=toks(4), block_ids=[0, 1, 2], drafts=toks(3)),
         dict(start=150, n=1, count=1, tokens=toks(1), block_ids=[3, 4, 5, 6, 7, 8, 9, 11, 12, 13], drafts=[]),
         dict(start=2, n=1, count=1, tokens=toks(1), block_ids=[10], drafts=[])],
    ]


def compare(shape):
    from types import SimpleNamespace

    from vllt.llama import LlamaRunner, fp32_reference_weights
    from vllt.runner import CudaRunner

    cache = SimpleNamespace(block_size=16, num_blocks=64)
    bf = LlamaRunner(shape, cache, max_seqs=8, max_tokens=256)
    ref = CudaRunner(shape, cache, max_seqs=8, max_tokens=256, weights=fp32_reference_weights(shape, bf.dev))
    rng = np.random.default_rng(3)
    worst, agree, rows, decided = 0.0, 0, 0, 0
    for seqs in schedule(shape.vocab_size, rng):
        out = F.as_scheduler_output(seqs)
        a, _ = bf.execute(out)
        b, _ = ref.execute(out)
        assert a.shape == b.shape and np.isfinite(a).all()
        err = np.abs(a - b).max()
        worst = max(worst, float(err / np.abs(b).max()))
        top2 = np.sort(b, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * err
        same = a.argmax(1) == b.argmax(1)
        assert same[clear].all(), "a row with a clear fp32 margin picked a different token"
        agree += int(same.sum())
        decided += int(clear.sum())
        rows += a.shape[0]
    return worst, agree / rows, decided


def test_bf16_small_llama_matches_fp32_rerun():
    from vllt.llama import LlamaShape

    shape = LlamaShape(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000,
                       max_seq_len=2048, seed=1)
    worst, agree, decided = compare(shape)
    print(f"small llama: max rel logit err {worst:.3e}, greedy agreement {agree:.2%}, {decided} clear rows")
    assert worst <= 5e-2


def test_bf16_llama8b_two_layer_slice_matches_fp32_rerun():
    from vllt.llama import LlamaShape

    shape = LlamaShape(n_layers=2, max_seq_len=2048)  # full width: d 4096, 32/8 heads, ffn 14336, vocab 128256
    worst, agree, decided = compare(shape)
    print(f"llama-8b 2-layer slice: max rel logit err {worst:.3e}, greedy agreement {agree:.2%}, "
          f"{decided} clear rows")
    assert worst <= 5e-2


def test_llama_engine_serves_requests_to_completion():
    """The bf16 runner behind the unmodified scheduler: chunked prefill, decode,
    every request reaches max_tokens, blocks all returned."""
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    from vllt.engine import gpu_engine
    from vllt.llama import LlamaRunner
    from vllt.workloads import llama_workload

    mc = ModelConfig(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000,
                     max_seq_len=2048, seed=1)
    cfg = EngineConfig(model=mc, cache=CacheConfig(block_size=16, num_blocks=512, enable_prefix_caching=False),
                       scheduler=SchedulerConfig(max_seqs=8, max_batched_tokens=256))
    eng = gpu_engine(cfg, runner_cls=LlamaRunner)
    reqs = llama_workload(12, seed=5, vocab=1000, prompt_mean=200, out_mean=20)
    for rid, ids, p in reqs:
        eng.add_request(params=p, request_id=rid, prompt_token_ids=[min(t, 999) for t in ids])
    while eng.has_work:
        eng.step()
    for rid, ids, p in reqs:
        assert len(eng.seqs[rid].output_token_ids) == p.max_tokens
    a = eng.scheduler.blocks.allocator
    assert a.num_free == a.num_blocks
