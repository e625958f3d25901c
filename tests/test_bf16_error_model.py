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
