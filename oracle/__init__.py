"""CPU oracle for the vllm-lite forward hot path. TEST INFRASTRUCTURE ONLY.

This package restates, in plain NumPy, the arithmetic of the reference
implementation (asp53826/vllm-lite, pure Python + NumPy) on the path that the
CUDA library replaces:

  attention.py  RoPE tables/rotation, block-table slot gather, K/V scatter,
                per-sequence paged attention      (vllmlite/attention.py:21-98)
  model.py      seeded TinyLlama weights and the batched forward pass
                                                   (vllmlite/model.py:17-120)
  runner.py     ModelRunner.execute batch flatten and copy-on-write
                                                   (vllmlite/runner.py:54-100)
  sampling.py   greedy / temperature / top-k / top-p sampling and the
                speculative accept/reject rule     (vllmlite/sampling.py:16-64,
                                                    vllmlite/speculative.py:86-100)
  llama_bf16.py the same forward with the bf16 Llama-shaped path's rounding
                points (torch on the CPU), to measure the bf16 error the GPU
                tests' tolerances are derived from; with rounding off it is
                pinned to model.py's forward

Who may use it: only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline
leg of `bench.py`, and only as the checker. The shipped library
(`vllm-lite_b200/vllt`) never imports it and has no CPU fallback.

Parity is pinned: `tests/golden/make_golden.py` runs the reference itself and
records its outputs; `tests/test_oracle_golden.py` checks every function here
against those fixtures.
"""
