"""Seeded request workloads for the benchmarks (host side, no device work).

`mixed_workload` restates the reference benchmark's generator
(bench/bench.py:35-47 and :152): lognormal prompt and output lengths clipped to
[16, 256] and [16, 192], prompt bytes uniform in [32, 126), a leading BOS (256)
and an optional shared prefix placed right after BOS. Drawing order and
arithmetic are kept so the requests are identical to the reference's for the
same seed (pinned by tests/golden/workload.npz).

`periodic_workload` is the speculative-decoding workload: each prompt is BOS
followed by a seeded token pattern of period 8..32 repeated to length 64..256.
The reference ships no generator for it; this one is ours.
"""

from __future__ import annotations

import numpy as np

BOS = 256


def _greedy_params(max_tokens: int):
    from vllmlite.sequence import SamplingParams

    return SamplingParams(max_tokens=int(max_tokens), temperature=0.0, ignore_eos=True)


def mixed_lengths(n: int, seed: int = 0, shared_prefix: int = 0, min_prompt: int = 16,
                  max_prompt: int = 256, min_out: int = 16, max_out: int = 192):
    """(prompt_token_ids, max_tokens) pairs, draw for draw like bench/bench.py:35-47."""
    rng = np.random.default_rng(seed)
    prefix = [int(t) for t in rng.integers(32, 126, size=shared_prefix)] if shared_prefix else []
    out = []
    for _ in range(n):
        plen = int(np.clip(rng.lognormal(np.log(min_prompt * 3), 0.6), min_prompt, max_prompt))
        olen = int(np.clip(rng.lognormal(np.log(min_out * 3), 0.7), min_out, max_out))
        body = [int(t) for t in rng.integers(32, 126, size=plen)]
        out.append(([BOS] + prefix + body, olen))
    return out


def mixed_workload(n: int = 48, seed: int = 0, shared_prefix: int = 0):
    """Requests as (request_id, prompt_token_ids, SamplingParams), greedy, ignore_eos."""
    return [(f"r{i}", ids, _greedy_params(m))
            for i, (ids, m) in enumerate(mixed_lengths(n, seed, shared_prefix))]


def periodic_lengths(n: int = 128, seed: int = 0, max_tokens: int = 256):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        period = int(rng.integers(8, 33))
        length = int(rng.integers(64, 257))
        pattern = rng.integers(32, 126, size=period)
        body = np.resize(pattern, length)
        out.append(([BOS] + [int(t) for t in body], max_tokens))
    return out


def periodic_workload(n: int = 128, seed: int = 0, max_tokens: int = 256):
    return [(f"p{i}", ids, _greedy_params(m))
            for i, (ids, m) in enumerate(periodic_lengths(n, seed, max_tokens))]


def llama_lengths(n: int = 512, seed: int = 0, vocab: int = 128256, prompt_mean: float = 1024,
                  out_mean: float = 256):
    """The Llama-3-8B-shaped serving workload: lognormal prompts (mean 1024,
    sigma 0.6, clipped to [32, 8192]) and outputs (mean 256, sigma 0.7, clipped
    to [16, 1024]); prompt tokens uniform over the vocabulary."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        plen = int(np.clip(rng.lognormal(np.log(prompt_mean) - 0.6 ** 2 / 2, 0.6), 32, 8192))
        olen = int(np.clip(rng.lognormal(np.log(out_mean) - 0.7 ** 2 / 2, 0.7), 16, 1024))
        out.append(([int(t) for t in rng.integers(0, vocab, size=plen)], olen))
    return out


def llama_workload(n: int = 512, seed: int = 0, **kw):
    return [(f"l{i}", ids, _greedy_params(m)) for i, (ids, m) in enumerate(llama_lengths(n, seed, **kw))]
