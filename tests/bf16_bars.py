#!/usr/bin/env python3
"""Measure the bf16 error that the GPU tests' tolerances are derived from.

    python tests/bf16_bars.py [--full]

Runs oracle/llama_bf16.py (the bf16 Llama-shaped forward's rounding points,
restated on the CPU) against its fp32 arithmetic on the schedules of
tests/test_gpu_llama.py and tests/tp_parity.py, for several weight seeds of
the product's N(0, 0.02) law, and prints per schedule the worst
(max-rel, row-rel) error of bf16 against fp32, of two tensor-parallel ranks
against one, of a planted mistake (one attention head zeroed), and (small
model) of the order of fp32 accumulation alone (float64 against fp32
contractions, both rounded at the bf16 points). The tests state their bars as
three times these measurements. --full adds the
full-width 2-layer slices (d 4096, vocabulary 128256: several minutes and
~20 GB of host memory).
"""

import argparse
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "vllm-lite_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--full", action="store_true")
    args = ap.parse_args()
    import torch

    from oracle.llama_bf16 import schedule_error
    from tests.test_gpu_llama import long_schedule, schedule
    from vllt.llama import LlamaShape

    torch.set_num_threads(os.cpu_count() or 1)
    runs = [("small", LlamaShape(n_layers=2, n_heads=8, n_kv_heads=2, d_model=1024, d_ff=2048, vocab_size=1000,
                                 max_seq_len=2048, seed=1), lambda v: schedule(v, np.random.default_rng(3)), 5)]
    if args.full:
        runs += [("full", LlamaShape(n_layers=2, max_seq_len=2048), lambda v: schedule(v, np.random.default_rng(3)), 2),
                 ("long", LlamaShape(n_layers=2, max_seq_len=9216),
                  lambda v: long_schedule(v, np.random.default_rng(8)), 1)]
    for name, shape, sched, seeds in runs:
        for seed in range(seeds):
            t = time.time()
            r = schedule_error(shape, sched(shape.vocab_size), seed=seed, tp=2, drop_head=5, order=name == "small")
            print(name, f"seed {seed}", {k: tuple(round(x, 5) for x in v) for k, v in r.items()},
                  f"{time.time() - t:.0f}s", flush=True)


if __name__ == "__main__":
    main()
