#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ by running the reference.

    python tests/golden/make_golden.py --reference <vllm-lite source checkout>

The reference (asp53826/vllm-lite, pure Python + NumPy) is imported from the
given source tree; nothing here is needed at test time. Outputs:

  weights.json      SHA-256 of every seeded weight array (vllmlite/model.py:47-62)
                    for the bench model and the small test model
  attention.npz     paged_attention outputs (vllmlite/attention.py:59) on the
                    reference's own test grid (tests/test_attention.py:36-57)
                    plus wider cases; inputs are regenerated from the seeds
  rope.npz          build_rope tables (vllmlite/attention.py:21)
  sampling.npz      sample() greedy path, _top_p keep sets, verify() results
  sampling_full.npz sample() temperature path with min_tokens EOS masks,
                    repetition penalties, top-k and top-p: the reference's
                    pick for a seeded generator, its uniform, keep set, probs
  workload.npz      make_workload requests (bench/bench.py:35-47) for the
                    mixed-length and shared-prefix benchmarks
  replay_*.npz      every ModelRunner.execute call of a reference LLMEngine run:
                    scheduler metadata in, logits out (vllmlite/runner.py:62-100)
  streams_*.npz     greedy output token streams of whole-engine runs
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root, for oracle/

# small test model used across the suites (2 layers, GQA 2, head_dim 16)
TINY = dict(n_layers=2, n_heads=4, n_kv_heads=2, d_model=64, d_ff=128, max_seq_len=512)
# the reference's published bench model (results/mixed_lengths.json args)
BENCH = dict(n_layers=6, n_heads=8, n_kv_heads=4, d_model=384, d_ff=1024, max_seq_len=512)

# prompts of our own for the engine-level streams
PROMPTS = [
    "paged attention keeps every sequence in fixed size blocks",
    "z",
    "continuous batching rebuilds the batch on every single forward pass, so",
    "kv",
    "a block table maps logical positions to physical cache blocks",
]
REPEATS = [
    "red green blue red green blue red green blue red green blue red green blue",
    "0123456789 0123456789 0123456789 0123456789 0123456789 0123456789",
]

# attention cases beyond the reference grid: (q_len, H, KV, D, block_size, ctx)
WIDE_ATTN = [
    (1, 8, 4, 48, 16, 1), (1, 8, 4, 48, 16, 15), (1, 8, 4, 48, 16, 16), (1, 8, 4, 48, 16, 17),
    (1, 8, 4, 48, 16, 300), (5, 8, 4, 48, 16, 300), (17, 8, 4, 48, 16, 64), (40, 8, 4, 48, 16, 40),
    (1, 32, 8, 128, 16, 257), (9, 32, 8, 128, 16, 129), (3, 4, 2, 16, 4, 23), (2, 8, 1, 64, 64, 130),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def attn_inputs(seed, q_len, H, KV, D, bs, ctx):
    """Inputs drawn exactly like tests/test_attention.py:40-53 of the reference
    (scattered block permutation, five spare blocks)."""
    rng = np.random.default_rng(seed)
    nb = (ctx + bs - 1) // bs
    total = nb + 5
    ck = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
    cv = rng.standard_normal((total * bs, KV, D)).astype(np.float32)
    bids = list(rng.permutation(total)[:nb])
    q = rng.standard_normal((q_len, H, D)).astype(np.float32)
    return q, ck, cv, bids


def capture_engine(LLMEngine, cfg, requests, spec_k=0):
    """Run a reference engine, recording every runner.execute call."""
    from vllmlite.speculative import NgramProposer

    eng = LLMEngine(cfg)
    if spec_k:
        eng.spec_k = spec_k
        eng.proposer = NgramProposer(spec_k)
    steps = []
    orig = eng.runner.execute

    def hooked(out):
        rec = {"cow": [tuple(map(int, p)) for p in out.cow], "seqs": []}
        for item in out.scheduled:
            s = item.seq
            start, n = item.start_pos, item.num_tokens
            rec["seqs"].append(dict(
                start=int(start), n=int(n), count=int(min(1 + len(s.draft_token_ids), n)),
                block_ids=[int(b) for b in s.table.block_ids],
                tokens=[int(t) for t in s.token_ids[start:start + n]],
                drafts=[int(t) for t in s.draft_token_ids]))
        logits, rows = orig(out)
        rec["logits"] = np.asarray(logits, np.float32).copy()
        rec["rows"] = [tuple(map(int, r)) for r in rows]
        steps.append(rec)
        return logits, rows

    eng.runner.execute = hooked
    ids = []
    for rid, toks, params in requests:
        ids.append(eng.add_request(params=params, request_id=rid, prompt_token_ids=toks))
    while eng.has_work:
        eng.step()
    streams = [list(eng.seqs[i].output_token_ids) for i in ids]
    return eng, steps, streams


def pack_steps(steps):
    """Flatten step records into int32/float32 arrays for an .npz."""
    meta, cow, logits, seq_rows = [], [], [], []
    toks, bids, drafts = [], [], []
    row0 = 0
    for si, st in enumerate(steps):
        for a, b in st["cow"]:
            cow.append((si, a, b))
        for s in st["seqs"]:
            seq_rows.append((si, s["start"], s["n"], s["count"], len(toks), len(s["tokens"]),
                             len(bids), len(s["block_ids"]), len(drafts), len(s["drafts"])))
            toks += s["tokens"]
            bids += s["block_ids"]
            drafts += s["drafts"]
        meta.append((si, row0, st["logits"].shape[0]))
        row0 += st["logits"].shape[0]
        logits.append(st["logits"])
    return dict(
        step_meta=np.asarray(meta, np.int32),
        seq_rows=np.asarray(seq_rows, np.int32),
        tokens=np.asarray(toks, np.int32),
        block_ids=np.asarray(bids, np.int32),
        drafts=np.asarray(drafts, np.int32).reshape(-1),
        cow=np.asarray(cow, np.int32).reshape(-1, 3),
        logits=np.concatenate(logits, 0).astype(np.float32),
    )


def streams_npz(streams):
    lens = np.asarray([len(s) for s in streams], np.int32)
    flat = np.asarray([t for s in streams for t in s], np.int16)
    return dict(lens=lens, tokens=flat)


def sampling_full():
    """Temperature rows through the reference's whole sampler
    (vllmlite/sampling.py:41-64): per row a logits vector, SamplingParams
    (temperature, top_k, top_p, min_tokens, repetition_penalty), the tokens
    seen so far, the number generated, and a seeded generator. Records the
    reference's pick, the uniform choice() drew (the generator's first
    random()), the keep set after mask / penalty / temperature / top-k /
    top-p (the reference's own private steps) and the final probabilities."""
    from vllmlite.sampling import _apply_repetition_penalty, _softmax, _top_k, _top_p, sample
    from vllmlite.sequence import SamplingParams

    rng = np.random.default_rng(11)
    V, N, eos = 261, 96, 257
    rows = (rng.standard_normal((N, V)) * 2.5).astype(np.float32)
    rows[3, eos] = rows[3].max() + 4.0  # EOS would win if it were not masked
    rows[7, 40] = rows[7, 41] = rows[7].max() + 0.5  # tie at the top
    params, seen_all, picks, us, keep, probs = [], [], [], [], [], []
    temps = (0.3, 0.7, 1.0, 1.6)
    for i in range(N):
        t = float(temps[i % 4])
        k = int((0, 0, 5, 40, 260, 261, 1000)[i % 7])
        p = float((1.0, 0.9, 0.5, 0.95, 0.2, 0.999)[i % 6])
        mint, ngen = int(i % 3) * 2, int(i % 5)
        pen = float((1.0, 1.3, 0.8, 2.0)[(i // 2) % 4])
        seen = [int(x) for x in rng.integers(0, V, size=int(rng.integers(0, 60)))]
        if i % 9 == 0:
            seen += [eos, eos]
        seed = 1000 + i
        prm = SamplingParams(temperature=t, top_k=k, top_p=p, min_tokens=mint, repetition_penalty=pen)
        picks.append(sample(rows[i], prm, seen, np.random.default_rng(seed), ngen, eos))
        us.append(np.random.default_rng(seed).random())
        x = rows[i].astype(np.float32, copy=True)
        if ngen < mint:
            x[eos] = -np.inf
        _apply_repetition_penalty(x, seen, pen)
        x /= t
        _top_k(x, k)
        _top_p(x, p)
        keep.append(np.isfinite(x))
        probs.append(_softmax(x).astype(np.float32))
        params.append((t, k, p, mint, ngen, pen, seed, len(seen)))
        seen_all += seen
    np.savez_compressed(
        os.path.join(HERE, "sampling_full.npz"), rows=rows, eos=np.int32(eos),
        params=np.asarray(params, np.float64), seen=np.asarray(seen_all, np.int32),
        picks=np.asarray(picks, np.int32), u=np.asarray(us, np.float64), keep=np.asarray(keep),
        probs=np.asarray(probs))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="vllm-lite source checkout")
    ap.add_argument("--skip-slow", action="store_true")
    ap.add_argument("--only", choices=["sampling_full"], help="write only this fixture")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    if args.only == "sampling_full":
        sampling_full()
        return

    from bench.bench import make_workload
    from vllmlite.attention import build_rope, gather_slots, paged_attention
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig
    from vllmlite.engine import LLMEngine
    from vllmlite.model import Layer, TinyLlama
    from vllmlite.sampling import _top_p, sample
    from vllmlite.sequence import SamplingParams
    from vllmlite.speculative import verify
    from vllmlite.tokenizer import ByteTokenizer

    t_all = time.time()

    # ---- weights -------------------------------------------------------------
    wj = {}
    for name, shape in (("tiny", TINY), ("bench", BENCH)):
        m = TinyLlama(ModelConfig(vocab_size=261, **shape))
        d = {"tok_emb": sha(m.tok_emb), "final_norm": sha(m.final_norm), "lm_head": sha(m.lm_head)}
        for i, layer in enumerate(m.layers):
            for k in Layer.__slots__:
                d[f"layers.{i}.{k}"] = sha(getattr(layer, k))
        wj[name] = {"shape": shape, "sha256": d, "num_params": int(m.num_params)}
    with open(os.path.join(HERE, "weights.json"), "w") as f:
        json.dump(wj, f, indent=1, sort_keys=True)

    # ---- rope ----------------------------------------------------------------
    rope = {}
    for D, P in ((8, 16), (16, 512), (48, 768), (128, 64)):
        c, s = build_rope(D, P)
        rope[f"cos_{D}_{P}"], rope[f"sin_{D}_{P}"] = c, s
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **rope)

    # ---- attention -------------------------------------------------------------
    cases, outs = [], {}
    seed = 0
    grid = [(q, h, kv, 8, bs, 37) for q in (1, 5, 17) for (h, kv) in ((4, 4), (8, 2), (6, 1))
            for bs in (1, 4, 16)]
    for (q_len, H, KV, D, bs, ctx) in grid + WIDE_ATTN:
        q, ck, cv, bids = attn_inputs(seed, q_len, H, KV, D, bs, ctx)
        slots = gather_slots(bids, bs, ctx)
        o = paged_attention(q, ck, cv, slots, KV, 1.0 / np.sqrt(D))
        outs[f"out_{len(cases)}"] = o.astype(np.float32)
        cases.append((seed, q_len, H, KV, D, bs, ctx))
        outs[f"insha_{len(cases) - 1}"] = np.frombuffer(
            bytes.fromhex(sha(q) + sha(ck)), np.uint8)
        seed += 1
    np.savez_compressed(os.path.join(HERE, "attention.npz"), cases=np.asarray(cases, np.int32),
                        **outs)

    # ---- sampling --------------------------------------------------------------
    rng = np.random.default_rng(7)
    V = 261
    rows = (rng.standard_normal((64, V)) * 3).astype(np.float32)
    rows[5, 17] = rows[5, 200] = rows[5].max() + 1  # a tie: first index must win
    ps = np.asarray([0.05, 0.3, 0.5, 0.9, 0.95, 0.999], np.float32)
    keep = np.zeros((len(rows), len(ps), V), bool)
    for i in range(len(rows)):
        for j, p in enumerate(ps):
            x = rows[i].copy()
            _top_p(x, float(p))
            keep[i, j] = np.isfinite(x)
    gtab, seen_all = [], []
    for i in range(len(rows)):
        seen = [int(t) for t in rng.integers(0, V, size=int(rng.integers(0, 40)))]
        pen = float([1.0, 1.3, 0.8][i % 3])
        mint, ngen = i % 4, i % 5
        prm = SamplingParams(temperature=0.0, min_tokens=mint, repetition_penalty=pen)
        picked = sample(rows[i], prm, seen, np.random.default_rng(0), ngen, 257)
        gtab.append((i, pen, mint, ngen, picked, len(seen)))
        seen_all += seen
    seen_flat = np.asarray(seen_all, np.int32)
    gtab = np.asarray(gtab, np.float64)
    vcases, vout = [], []
    for i in range(48):
        k = int(rng.integers(1, 9))
        picks = rng.integers(0, 12, size=k + 1)
        lg = np.full((k + 1, 12), -5.0, np.float32)
        lg[np.arange(k + 1), picks] = 5.0
        lg += (rng.standard_normal(lg.shape) * 0.1).astype(np.float32)
        drafts = [int(picks[j]) if rng.random() < 0.7 else int(rng.integers(0, 12)) for j in range(k)]
        toks, acc = verify(lg, drafts)
        vcases.append((lg, drafts, toks, acc))
    np.savez_compressed(
        os.path.join(HERE, "sampling.npz"), rows=rows, top_p=ps, keep=keep,
        greedy=gtab, greedy_seen=seen_flat,
        verify_logits=np.concatenate([c[0] for c in vcases]),
        verify_k=np.asarray([len(c[1]) for c in vcases], np.int32),
        verify_drafts=np.asarray([d for c in vcases for d in c[1]], np.int32),
        verify_tokens=np.asarray([t for c in vcases for t in c[2]], np.int32),
        verify_ntok=np.asarray([len(c[2]) for c in vcases], np.int32),
        verify_accepted=np.asarray([c[3] for c in vcases], np.int32))
    sampling_full()

    # ---- workloads -------------------------------------------------------------
    wl = {}
    for name, prefix, maxlen in (("mixed", 0, 512), ("shared", 256, 768)):
        reqs = make_workload(48, np.random.default_rng(0), 16, 256, 16, 192, prefix)
        wl[f"{name}_lens"] = np.asarray([len(r[1]) for r in reqs], np.int32)
        wl[f"{name}_tokens"] = np.asarray([t for r in reqs for t in r[1]], np.int16)
        wl[f"{name}_max_tokens"] = np.asarray([r[2].max_tokens for r in reqs], np.int32)
    np.savez_compressed(os.path.join(HERE, "workload.npz"), **wl)

    def engine_cfg(shape, bs=16, nb=512, max_seqs=8, budget=1024, prefix=False, maxlen=None):
        mc = ModelConfig(vocab_size=261, **shape)
        if maxlen:
            mc.max_seq_len = maxlen
        return EngineConfig(model=mc,
                            cache=CacheConfig(block_size=bs, num_blocks=nb, enable_prefix_caching=prefix),
                            scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget))

    tok = ByteTokenizer()

    def reqs_of(prompts, max_tokens):
        p = SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True)
        return [(f"q{i}", tok.encode(x), p) for i, x in enumerate(prompts)]

    # ---- replays: every execute() call, metadata in, logits out -----------------
    t = time.time()
    # bench model, chunked prefill (budget 96), 4 seats, block 16
    _, steps, _ = capture_engine(LLMEngine, engine_cfg(BENCH, max_seqs=4, budget=96),
                                 reqs_of(PROMPTS, 10))
    np.savez_compressed(os.path.join(HERE, "replay_bench.npz"), **pack_steps(steps))
    # bench model, speculative k=4 on repeating prompts, prefix cache, block 4
    shared = "the shared system prompt of every request: "
    _, steps, _ = capture_engine(
        LLMEngine, engine_cfg(BENCH, bs=4, nb=512, max_seqs=4, budget=256, prefix=True),
        reqs_of([shared + r for r in REPEATS] + [shared + "x"], 24), spec_k=4)
    np.savez_compressed(os.path.join(HERE, "replay_spec.npz"), **pack_steps(steps))
    print(f"replays {time.time() - t:.1f}s")

    # ---- streams ----------------------------------------------------------------
    t = time.time()
    _, _, s_tiny = capture_engine(LLMEngine, engine_cfg(TINY), reqs_of(PROMPTS, 20))
    _, _, s_rep = capture_engine(LLMEngine, engine_cfg(TINY), reqs_of(REPEATS, 40))
    np.savez_compressed(os.path.join(HERE, "streams_tiny.npz"),
                        **{f"prompts_{k}": v for k, v in streams_npz(s_tiny).items()},
                        **{f"repeats_{k}": v for k, v in streams_npz(s_rep).items()})
    print(f"tiny streams {time.time() - t:.1f}s")
    if not args.skip_slow:
        for name, prefix, maxlen in (("mixed", 0, 512), ("shared", 256, 768)):
            t = time.time()
            reqs = make_workload(48, np.random.default_rng(0), 16, 256, 16, 192, prefix)
            nb = 16 * maxlen // 16
            eng, _, s = capture_engine(LLMEngine, engine_cfg(
                BENCH, nb=nb, max_seqs=16, budget=1024, prefix=bool(prefix), maxlen=maxlen), reqs)
            st = eng.stats()
            np.savez_compressed(os.path.join(HERE, f"streams_{name}.npz"),
                                steps=np.int32(st["steps"]), **streams_npz(s))
            print(f"{name} streams {time.time() - t:.1f}s steps={st['steps']}")
        # periodic prompts for the speculative benchmark (k=0 is the truth)
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "vllm-lite_b200"))
        from vllt.workloads import periodic_workload

        t = time.time()
        reqs = periodic_workload(128, seed=0)
        eng, _, s = capture_engine(LLMEngine, engine_cfg(
            BENCH, nb=4096, max_seqs=64, budget=2048, maxlen=1024), reqs)
        np.savez_compressed(os.path.join(HERE, "streams_periodic.npz"),
                            steps=np.int32(eng.stats()["steps"]), **streams_npz(s))
        print(f"periodic streams {time.time() - t:.1f}s")
    print(f"done in {time.time() - t_all:.1f}s")


if __name__ == "__main__":
    main()
