"""CPU: the error model behind the bf16 GPU tests' tolerances.

oracle/llama_bf16.py restates the bf16 Llama-shaped forward's rounding points
on the CPU. The GPU tests (tests/test_gpu_llama.py, tests/tp_parity.py) state
their bars as three times the worst error it measures; this test re-measures
the small model's schedule and checks that the bars still hold that margin,
and that a planted mistake in the oracle (one attention head zeroed in every
layer) lands far outside them.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def test_bars_are_three_times_the_measured_bf16_error():
    from oracle.llama_bf16 import schedule_error
    from tests.test_gpu_llama import SMALL_BAR, schedule
    from tests.tp_parity import TP_BAR
    from vllt.llama import LlamaShape

    shape = LlamaShape(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000,
                       max_seq_len=2048, seed=1)
    for seed in (0, 1):
        r = schedule_error(shape, schedule(shape.vocab_size, np.random.default_rng(3)), seed=seed, tp=2,
                           drop_head=5)
        assert 1e-3 < max(r["bf16"]) and 3 * max(r["bf16"]) <= SMALL_BAR, r
        assert 3 * max(r["tp"]) <= TP_BAR, r
        assert min(r["dropped"]) > 5 * SMALL_BAR, r


def test_error_model_computes_the_reference_forward_without_rounding():
    """With rounding off, oracle/llama_bf16.py is the reference's forward
    (vllmlite/model.py:80-120, as oracle/model.py restates it and the golden
    replays pin it): same RoPE pairs, GQA head grouping, SwiGLU and norms, on
    the reference's seeded weights of a small model; logits at every position
    agree within fp32 reassociation."""
    from oracle import model as OM
    from oracle.llama_bf16 import forward_sequence
    from tests import fixtures as F

    cfg = OM.Shape(vocab_size=261, **F.TINY)
    w = OM.seeded_weights(cfg)
    emu = {"tok_emb": torch.from_numpy(w["tok_emb"]), "lm_head": torch.from_numpy(w["lm_head"].T.copy())}
    for i in range(cfg.n_layers):
        for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
            emu[f"{i}.{k}"] = torch.from_numpy(w[f"layers.{i}.{k}"].T.copy())  # reference [in][out] -> [out][in]
    T = 37
    toks = np.random.default_rng(2).integers(0, 261, size=T)
    hd, KV = cfg.head_dim, cfg.n_kv_heads
    ck = np.zeros((cfg.n_layers, T, KV, hd), np.float32)
    cv = np.zeros_like(ck)
    slots = np.arange(T)
    want = OM.forward(cfg, w, toks, np.arange(T), ck, cv, [(0, T, slots, slots)], np.arange(T))
    with torch.no_grad():
        got = forward_sequence(cfg, emu, toks.tolist(), [(0, T)], bf16=False).numpy()
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5 * np.abs(want).max())
