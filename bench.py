#!/usr/bin/env python3
"""Benchmark of the vllt forward hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload mixed|shared|decode]
    python bench.py --impl reference ...      (the reference's NumPy engine on host cores)

Default workload "mixed" is the reference's headline benchmark
(bench/bench.py of vllm-lite, results/mixed_lengths.json): 48 greedy requests,
lognormal prompt/output lengths, 6 layers / d_model 384 / 8 heads / 4 KV heads /
d_ff 1024 / vocab 261, fp32, block 16, 512 blocks, max_seqs 16, token budget
1024, random-init weights from the reference seed (synthetic data). One bench
step = the whole 48-request workload pushed through the engine.
  value   engine output tok/s with device-side token picks (GpuLLMEngine)
  e2e     the same through the reference-facing drop-in: an unmodified
          LLMEngine whose runner is CudaRunner, logits copied to the host
Also measured in the same run: TTFT p50, and the paged-attention decode
kernel on the decode microbenchmark (256 sequences, contexts U[1,4096],
32 / 8 heads, head_dim 128, bf16, block 16) as achieved HBM GB/s -> "roofline".

With --gpus N (torchrun, one process per GPU) every rank runs an independent
engine replica on its own seeded workload (the path has no data-parallel
exchange), "scaling": "weak", value = total tokens / max elapsed over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "vllm-lite_b200"), os.path.join(ROOT, "baseline", "_ref")):
    if os.path.isdir(p) and p not in sys.path:
        sys.path.insert(0, p)

PUBLISHED = {"mixed": 2028.0, "shared": 1288.6}  # reference README / results/*.json (M-series CPU)
MODEL = dict(n_layers=6, n_heads=8, n_kv_heads=4, d_model=384, d_ff=1024)


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def engine_config(workload: str):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    shared = workload == "shared"
    maxlen = 768 if shared else 512
    mc = ModelConfig(vocab_size=261, max_seq_len=maxlen, **MODEL)
    # the reference bench's KV budget: max_seqs * max_len slots (bench/bench.py:156-157)
    return EngineConfig(model=mc,
                        cache=CacheConfig(block_size=16, num_blocks=16 * maxlen // 16, enable_prefix_caching=shared),
                        scheduler=SchedulerConfig(max_seqs=16, max_batched_tokens=1024))


def requests(workload: str, seed: int):
    from vllt.workloads import mixed_workload

    return mixed_workload(48, seed, 256 if workload == "shared" else 0)


def run_workload(eng, reqs, tag, nvtx_window=None):
    """Submit every request, drive step() until drained (bench/bench.py:83-88).
    nvtx_window=(a, b): steps a..b-1 of this run sit in an NVTX range
    "vllt_window" (for `ncu --nvtx --nvtx-include vllt_window/`)."""
    for rid, ids, params in reqs:
        eng.add_request(params=params, request_id=f"{tag}-{rid}", prompt_token_ids=ids)
    steps0 = eng.total_steps
    while eng.has_work:
        i = eng.total_steps - steps0
        if nvtx_window and i == nvtx_window[0]:
            import torch

            torch.cuda.nvtx.range_push("vllt_window")
        eng.step()
        if nvtx_window and i == nvtx_window[1] - 1:
            import torch

            torch.cuda.nvtx.range_pop()
    seqs = [eng.seqs[f"{tag}-{rid}"] for rid, _, _ in reqs]
    out_tokens = sum(len(s.output_token_ids) for s in seqs)
    lat = {k: [getattr(s, k) for s in seqs if getattr(s, k) is not None] for k in ("ttft", "tpot", "e2e")}
    for rid, _, _ in reqs:
        eng.release(f"{tag}-{rid}")
    return out_tokens, lat, eng.total_steps - steps0


def merge_latency(lats):
    """Per-request latency lists (ttft / tpot / e2e, seconds) of several runs, joined."""
    return {k: [x for lat in lats for x in lat[k]] for k in ("ttft", "tpot", "e2e")}


def latency_summary(lat, digits: int = 2):
    """p50 / p99 in ms of time to first token, time per output token after the
    first, and request latency, with the reference bench's percentile
    (numpy's, bench/bench.py:30-32, :61-66)."""
    out = {}
    for k in ("ttft", "tpot", "e2e"):
        for q in (50, 99):
            out[f"{k}_p{q}_ms"] = round(1e3 * float(np.percentile(lat[k], q)), digits) if lat[k] else None
    return out


class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


def flush_l2(torch, dev):
    """Write 256 MB (> the 126 MB L2) between timed iterations."""
    buf = getattr(flush_l2, "buf", None)
    if buf is None:
        buf = flush_l2.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    buf.zero_()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---- decode microbenchmark (the paged-attention roofline) ---------------------------------
def decode_setup(torch, dev, seqs=256, H=32, KV=8, D=128, bs=16, seed=0, max_ctx=4096):
    import numpy as np

    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, max_ctx + 1, size=seqs)
    nblk = (ctx + bs - 1) // bs
    pool = int(nblk.sum()) + 64
    perm = rng.permutation(pool)
    W = int(nblk.max())
    tables = np.zeros((seqs, W), np.int32)
    o = 0
    for i, n in enumerate(nblk):
        tables[i, :n] = perm[o:o + n]
        o += n
    g = torch.Generator(device=dev).manual_seed(seed)
    kc = torch.randn((pool, KV, bs, D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn((pool, KV, bs, D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((seqs, H, D), generator=g, device=dev).to(torch.bfloat16)
    knew = torch.randn((seqs, KV, D), generator=g, device=dev).to(torch.bfloat16)
    vnew = torch.randn((seqs, KV, D), generator=g, device=dev).to(torch.bfloat16)
    last = ctx - 1
    slots = tables[np.arange(seqs), last // bs] * bs + last % bs
    sum_ctx = int(ctx.sum())
    alg_bytes = (sum_ctx * KV * D * 2 * 2          # K and V read
                 + 2 * seqs * H * D * 2            # Q read, O written
                 + 2 * seqs * KV * D * 2 * 2       # new K/V read and written
                 + int(nblk.sum()) * 4)            # block tables
    return dict(kc=kc, vc=vc, q=q, knew=knew, vnew=vnew, tables=torch.from_numpy(tables).to(dev),
                cu=torch.arange(seqs + 1, dtype=torch.int32, device=dev),
                ctx=torch.from_numpy(ctx.astype(np.int32)).to(dev), slots=torch.from_numpy(slots.astype(np.int32)).to(dev),
                seqs=seqs, H=H, KV=KV, D=D, bs=bs, pool=pool, W=W, max_ctx=int(ctx.max()), sum_ctx=sum_ctx,
                alg_bytes=alg_bytes, attn_bytes=sum_ctx * KV * D * 4 + 2 * seqs * H * D * 2 + int(nblk.sum()) * 4)


def decode_write(s):
    """One new token per sequence into the paged cache (reshape_and_cache)."""
    from vllt import _lib

    L = _lib.lib()
    _lib.check(L.vllt_reshape_and_cache(s["knew"].data_ptr(), s["vnew"].data_ptr(), s["kc"].data_ptr(),
                                        s["vc"].data_ptr(), s["slots"].data_ptr(), s["seqs"], s["KV"], s["D"],
                                        s["bs"], s["pool"], _lib.VLLT_BF16, _lib.stream_handle()))


def decode_attend(s, ws, out):
    """Single-query paged attention over every sequence (TMA decode kernel + split merge)."""
    from vllt import _lib

    L = _lib.lib()
    _lib.check(L.vllt_paged_attention_varlen(
        s["q"].data_ptr(), s["kc"].data_ptr(), s["vc"].data_ptr(), s["tables"].data_ptr(), s["W"],
        s["cu"].data_ptr(), s["ctx"].data_ptr(), s["seqs"], s["seqs"], 1, s["max_ctx"], s["H"], s["KV"], s["D"],
        s["bs"], s["pool"], float(1.0 / s["D"] ** 0.5), _lib.VLLT_BF16, out.data_ptr(), ws.data_ptr(),
        ws.numel(), _lib.stream_handle()))


def decode_bench(torch, dev, steps, warmup):
    """Time K decode steps (cache write + attention) with CUDA events on the
    launching stream, L2 flushed before each; the attention call is bracketed
    by its own events for the roofline. Returns (setup, step s, attention s)."""
    from vllt import _lib

    s = decode_setup(torch, dev)
    nbytes = _lib.lib().vllt_attention_workspace_bytes(s["seqs"], s["H"], s["D"], s["max_ctx"])
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(s["q"])
    for _ in range(max(warmup, 3)):
        decode_write(s)
        decode_attend(s, ws, out)
    torch.cuda.synchronize()
    step_t, attn_t = [], []
    torch.cuda.nvtx.range_push("vllt_decode")  # ncu --nvtx --nvtx-include vllt_decode/
    for _ in range(max(steps, 5)):
        flush_l2(torch, dev)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        decode_write(s)
        e1.record()
        decode_attend(s, ws, out)
        e2.record()
        e2.synchronize()
        step_t.append(e0.elapsed_time(e2) / 1e3)
        attn_t.append(e1.elapsed_time(e2) / 1e3)
    torch.cuda.nvtx.range_pop()
    if int(ws[:4].view(torch.int32).item()) != 0:
        raise RuntimeError("decode attention reported a device-side timeout")
    return s, statistics.median(step_t), statistics.median(attn_t)


# ---- our arm -------------------------------------------------------------------------------
def main_ours(args):
    import numpy as np
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from vllt import _lib
    from vllt.engine import cuda_engine, gpu_engine

    L = _lib.lib()
    wl = args.workload
    if wl == "decode":
        return main_decode(args, torch, dev, rank, world)
    if wl == "llama8b":
        return main_llama(args, torch, dev, rank, world)
    if wl == "spec":
        return main_spec(args, torch, dev, rank, world)
    if wl == "gemm":
        return main_gemm(args, torch, dev, rank, world)
    if wl == "prefill":
        return main_prefill(args, torch, dev, rank, world)
    cfg = engine_config(wl)
    reqs = requests(wl, seed=rank)  # each replica its own seeded workload
    eng = gpu_engine(cfg)
    ref_eng = cuda_engine(engine_config(wl))
    # warm-up: whole workloads through both engines (graphs of allocations, caches)
    for i in range(args.warmup):
        run_workload(eng, reqs, f"w{i}")
    run_workload(ref_eng, reqs, "w")

    window = tuple(int(x) for x in args.nvtx_passes.split(":")) if args.nvtx_passes else None

    def timed(engine, tag, nvtx_window=None):
        flush_l2(torch, dev)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        run = engine.runner

        def launched():  # kernels executed: direct launches + graph replays - capture-time calls
            return L.vllt_kernel_launches() + run.replayed_kernels - run.captured_kernels

        l0 = launched()
        e0.record()
        toks, lat, steps = run_workload(engine, reqs, tag, nvtx_window)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3, toks, lat, steps, launched() - l0

    res = []
    torch.cuda.nvtx.range_push("vllt_timed")  # ncu --nvtx --nvtx-include vllt_timed/
    with Clocks(local) as clk:
        for i in range(args.steps):
            res.append(timed(eng, f"t{i}", window if i == 0 else None))
    torch.cuda.nvtx.range_pop()
    e2e_res = [timed(ref_eng, f"e{i}") for i in range(max(1, min(args.steps, 3)))]
    # untimed extra run: per-pass GPU time (CUDA events around each forward) vs the rest of a step
    eng.runner.pass_log = []
    flush_l2(torch, dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ahead0 = eng.passes_ahead
    e0.record()
    run_workload(eng, reqs, "b")
    e1.record()
    torch.cuda.synchronize()
    ps = eng.runner.pass_summary()
    eng.runner.pass_log = None
    # host_and_other_s: the run's time outside forward passes (the GPU idles
    # or runs the pick kernels); passes_ahead: passes launched while the
    # previous pass still ran (the engine's run-ahead)
    breakdown = dict(ps, run_s=round(e0.elapsed_time(e1) / 1e3, 4),
                     host_and_other_s=round(e0.elapsed_time(e1) / 1e3 - ps["gpu_s"], 4),
                     passes_ahead=eng.passes_ahead - ahead0)
    # H2D / D2H bytes of one workload pass through the drop-in runner
    rr = ref_eng.runner
    t_ours = sum(r[0] for r in res)
    toks = sum(r[1] for r in res)
    t_e2e = sum(r[0] for r in e2e_res)
    toks_e2e = sum(r[1] for r in e2e_res)
    if world > 1:
        import torch.distributed as dist

        v = torch.tensor([t_ours, t_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        n = torch.tensor([toks, toks_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
        t_ours, t_e2e = float(v[0]), float(v[1])
        toks, toks_e2e = float(n[0]), float(n[1])
    lat_all = merge_latency([r[2] for r in res])
    decode_s, _, decode_t = decode_bench(torch, dev, 10, 3)
    hbm, peak_kind = peaks()
    achieved = decode_s["attn_bytes"] / decode_t / 1e9  # attention bytes / attention-call time
    cpu = cpu_baseline(wl) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    steps_per_run = res[0][3]
    launches = res[0][4]
    line = {
        "metric": "engine output tok/s (48-request mixed-length greedy workload)" if wl == "mixed"
        else "engine output tok/s (48-request shared-prefix workload, prefix cache on)",
        "value": round(toks / t_ours, 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * t_ours / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(toks / t_ours / world / PUBLISHED[wl], 3),
        "dtype": "f32",
        "data": "synthetic (reference-seeded random weights and seeded request generator)",
        "impl": "vllt",
        "config": {"workload": f"C1 {wl}: 48 requests, 6L/384d/8H/4KV/d_ff1024/V261 fp32, block 16, "
                               f"max_seqs 16, budget 1024" + (", 256-token shared prefix" if wl == "shared" else ""),
                   "model": "TinyLlama-style 6L/384d (vllm-lite bench model)", "global_batch": 48 * world,
                   "seq_len": 768 if wl == "shared" else 512, "parallelism": f"replicas x{world}",
                   "forward_passes_per_step": steps_per_run, "l2": "flushed (256 MB write) before each timed step"},
        **latency_summary(lat_all),
        "e2e": {"value": round(toks_e2e / t_e2e, 1), "unit": "tok/s",
                "api": "vllmlite LLMEngine + vllt.CudaRunner (host logits)",
                "h2d_bytes_per_step": int(rr.h2d_bytes / max(rr.steps, 1) * steps_per_run),
                "d2h_bytes_per_step": int(rr.d2h_bytes / max(rr.steps, 1) * steps_per_run)},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "paged-attention decode (256 seqs, ctx U[1,4096], 32/8 heads, D128, bf16)",
                     "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "peak_kind": peak_kind,
                     "unit": "GB/s", "frac": round(achieved / hbm, 3),
                     "bytes_per_launch": decode_s["attn_bytes"], "sum_ctx": decode_s["sum_ctx"],
                     "launch_ms": round(decode_t * 1e3, 4), "traffic": None,
                     "traffic_note": "no ncu capture of the current decode kernel; the earlier version with "
                                     "the same access pattern read 2.254 GB + wrote 0.014 GB per launch "
                                     "(= algorithmic)"},
        "clocks": clk.summary(),
        "breakdown": breakdown,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def spec_config():
    """C5: the bench model with room for 257-token prompts + 256 outputs."""
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    mc = ModelConfig(vocab_size=261, max_seq_len=1024, **MODEL)
    return EngineConfig(model=mc, cache=CacheConfig(block_size=16, num_blocks=4096, enable_prefix_caching=False),
                        scheduler=SchedulerConfig(max_seqs=64, max_batched_tokens=2048))


def main_spec(args, torch, dev, rank, world):
    """C5: 128 periodic prompts, 256 greedy tokens each, n-gram speculation with
    k drafts verified on the device; token streams must equal k = 0."""
    from vllt import _lib
    from vllt.engine import gpu_engine
    from vllt.workloads import periodic_workload

    L = _lib.lib()
    k = args.spec_k
    reqs = periodic_workload(128, seed=rank)

    def streams(eng, tag):
        return [list(eng.seqs[f"{tag}-{rid}"].output_token_ids) for rid, _, _ in reqs]

    base = gpu_engine(spec_config(), speculative_tokens=0)
    eng = gpu_engine(spec_config(), speculative_tokens=k)
    for i in range(args.warmup):
        run_workload(eng, reqs, f"w{i}")
    # identity against k = 0 (outputs read before release)
    for rid, ids, params in reqs:
        base.add_request(params=params, request_id=f"b-{rid}", prompt_token_ids=ids)
        eng.add_request(params=params, request_id=f"c-{rid}", prompt_token_ids=ids)
    while base.has_work:
        base.step()
    while eng.has_work:
        eng.step()
    same = streams(base, "b") == streams(eng, "c")
    eng.spec.proposed = eng.spec.accepted = 0
    ts, toks, lats, launches = [], 0, [], 0
    run = eng.runner
    with Clocks(int(os.environ.get("LOCAL_RANK", 0))) as clk:
        for i in range(args.steps):
            flush_l2(torch, dev)
            torch.cuda.synchronize()
            l0 = L.vllt_kernel_launches() + run.replayed_kernels - run.captured_kernels
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            n, lat, _ = run_workload(eng, reqs, f"t{i}")
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
            launches = L.vllt_kernel_launches() + run.replayed_kernels - run.captured_kernels - l0
            toks += n
            lats.append(lat)
    t = sum(ts)
    if world > 1:
        import torch.distributed as dist

        v = torch.tensor([t, toks], device=dev, dtype=torch.float64)
        dist.all_reduce(v[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(v[1:], op=dist.ReduceOp.SUM)
        t, toks = float(v[0]), float(v[1])
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = spec_cpu_baseline(k)
    if rank == 0:
        line = {
            "metric": f"engine output tok/s (C5: 128 periodic prompts, speculative k={k})",
            "value": round(toks / t, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "vllt",
            "data": "synthetic (reference-seeded weights, seeded periodic prompts)",
            "config": {"workload": f"C5: 128 periodic prompts (period 8-32, length 64-256), 256 greedy tokens, "
                                   f"n-gram proposer k={k}, 6L/384d fp32, max_seqs 64, budget 2048",
                       "parallelism": f"replicas x{world}", "l2": "flushed before each timed step"},
            "token_identical_to_k0": bool(same),
            "acceptance": round(eng.spec.accepted / max(eng.spec.proposed, 1), 4),
            **latency_summary(merge_latency(lats)),
            "gpu_launches": int(launches), "e2e": None, "clocks": clk.summary()}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def spec_cpu_baseline(k: int, n: int = 16):
    """The unmodified reference engine (NumpyRunner, LLMEngine(speculative_tokens=k))
    on the first n of the same periodic prompts: a bounded sample."""
    try:
        from vllmlite.engine import LLMEngine
    except Exception as e:  # pragma: no cover
        return {"value": None, "unit": "tok/s", "unavailable": f"vllm-lite not importable: {e}"}
    from vllt.workloads import periodic_workload

    reqs = periodic_workload(128, seed=0)[:n]
    eng = LLMEngine(spec_config(), speculative_tokens=k)
    run_workload(eng, reqs[:2], "cw")  # warm-up
    t0 = time.perf_counter()
    toks, _, _ = run_workload(eng, reqs, "c")
    dt = time.perf_counter() - t0
    return {"value": round(toks / dt, 1), "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
            "sample": f"first {n} of the 128 periodic prompts, 256 tokens each, vllm-lite LLMEngine("
                      f"speculative_tokens={k}) with NumpyRunner, after a 2-request warm-up"}


def _tc_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def _event_times(torch, fn, steps, warmup, dev):
    """Median CUDA-event seconds of fn() over max(steps, 3) launches, L2
    flushed before each, after max(warmup, 3) untimed launches."""
    for _ in range(max(warmup, 3)):
        fn()
    ts = []
    for _ in range(max(steps, 3)):
        flush_l2(torch, dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) / 1e3)
    return statistics.median(ts)


def _graph_time(torch, fns, reps):
    """Seconds per call of fns (cycled), captured back to back in one CUDA graph
    and replayed: no host launch latency inside the timed region. Median of
    max(reps, 3) replays, L2 flushed before each."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    ts = []
    for _ in range(max(reps, 3)):
        flush_l2(torch, torch.device("cuda", torch.cuda.current_device()))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) / 1e3)
    del g
    return statistics.median(ts) / len(fns)


def main_gemm(args, torch, dev, rank, world):
    """tcgen05 bf16 GEMM on the Llama-3-8B projection shapes, prefill (M=8192)
    and decode (M=512, 256, 64) batches: TFLOP/s against the measured cuBLAS
    bf16 peak, and weight GB/s for the decode batches. Each shape runs in the
    form the forward pass picks for it ("splits" 0 = small-M stream-K form).
    Launches are timed inside a CUDA graph (as the forward runs them), cycling
    over enough weight copies that the weights of consecutive launches do not
    fit in L2 together, like consecutive layers."""
    from vllt import _lib

    L = _lib.lib()
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    shapes = [("qkv", 6144, 4096), ("o_proj", 4096, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336)]
    if args.gemm_shape:
        shapes = [x for x in shapes if x[0] in args.gemm_shape.split(",")]
    peak, kind = _tc_peak()
    hbm, _ = peaks()
    res = {}
    tot_flops = tot_t = 0.0
    ms = [int(x) for x in args.gemm_m.split(",")] if args.gemm_m else [8192, 512, 256, 64]
    for M in ms:
        A = torch.randn((M, 14336), device=dev).to(torch.bfloat16)
        for name, N, K in shapes:
            copies = max(2, -(-320 * 2 ** 20 // (N * K * 2)))
            Ws = [torch.randn((N, K), device=dev).to(torch.bfloat16) for _ in range(copies)]
            C_ = torch.empty((M, N), device=dev)
            a = A[:, :K].contiguous()
            splits = int(L.vllt_gemm_bf16_auto_splits(M, N, K))
            ws = torch.zeros(max(int(L.vllt_gemm_bf16_splitk_workspace_bytes(M, N, K, splits)), 256),
                             dtype=torch.uint8, device=dev)

            def launcher(W):
                def run():
                    _lib.check(L.vllt_gemm_bf16_splitk(a.data_ptr(), W.data_ptr(), C_.data_ptr(), M, N, K, splits,
                                                       ws.data_ptr(), ws.numel(), flags.data_ptr(),
                                                       _lib.stream_handle()))
                return run
            fns = [launcher(W) for W in Ws] * max(1, 8 // copies)
            for f in fns:  # untimed, outside capture: first-use setup
                f()
            t = _graph_time(torch, fns, args.steps)
            # cuBLAS on the same operands and launch pattern, as a reference point only
            outs = [torch.empty((M, N), device=dev, dtype=torch.bfloat16) for _ in Ws]

            def lib_launcher(W, o):
                def run():
                    torch.matmul(a, W.t(), out=o)
                return run
            lib_fns = [lib_launcher(W, o) for W, o in zip(Ws, outs)] * max(1, 8 // copies)
            for f in lib_fns:
                f()
            t_lib = _graph_time(torch, lib_fns, args.steps)
            fl = 2.0 * M * N * K
            res[f"M{M}_{name}"] = {"tflops": round(fl / t / 1e12, 1), "us": round(t * 1e6, 2), "splits": splits,
                                   "tc_frac": round(fl / t / 1e12 / peak, 3),
                                   "weight_gbs": round(N * K * 2 / t / 1e9, 1),
                                   "hbm_frac": round(N * K * 2 / t / 1e9 / hbm, 3),
                                   "cublas_us": round(t_lib * 1e6, 2)}
            del outs
            if M == 8192:
                tot_flops += fl
                tot_t += t
            del Ws, C_, ws
    assert int(flags.item()) == 0, "bounded wait expired in the GEMM"
    if rank == 0:
        v = tot_flops / tot_t / 1e12 if tot_t else 0.0
        print(json.dumps({"metric": "tcgen05 bf16 GEMM TFLOP/s (Llama-3-8B projections, M=8192)", "value": round(v, 1),
                          "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic N(0,1)",
                          "config": {"workload": "the four GEMM shapes of one Llama-3-8B layer",
                                     "timing": "CUDA graph of 8 launches over rotating weight copies",
                                     "l2": "flushed before each replay; weights of consecutive launches exceed L2"},
                          "roofline": {"bound": "tensor", "achieved": round(v, 1), "peak": peak, "unit": "TFLOP/s",
                                       "frac": round(v / peak, 3), "peak_kind": kind, "traffic": None},
                          "shapes": res}), flush=True)


def main_prefill(args, torch, dev, rank, world):
    """tcgen05 prefill attention: 16 sequences x 2048-token prompts (causal),
    32 / 8 heads, head_dim 128, bf16, block 16; FLOPs = 4 * D * H per causal
    (query, key) pair."""
    import numpy as np

    from vllt import _lib

    L = _lib.lib()
    S, P, H, KV, D, bs = 16, 2048, 32, 8, 128, 16
    nb = S * P // bs
    rng = np.random.default_rng(0)
    tables = torch.from_numpy(rng.permutation(nb).astype(np.int32).reshape(S, P // bs)).to(dev)
    kc = torch.randn((nb, KV, bs, D), device=dev).to(torch.bfloat16)
    vc = torch.randn((nb, KV, bs, D), device=dev).to(torch.bfloat16)
    q = torch.randn((S * P, H, D), device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    cu = torch.arange(0, S * P + 1, P, dtype=torch.int32, device=dev)
    ctx = torch.full((S,), P, dtype=torch.int32, device=dev)
    ws = torch.zeros(max(L.vllt_attention_workspace_bytes(S, H, D, P), 256), dtype=torch.uint8, device=dev)

    def run():
        _lib.check(L.vllt_paged_attention_varlen(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(),
                                                 P // bs, cu.data_ptr(), ctx.data_ptr(), S, S * P, P, P, H, KV, D,
                                                 bs, nb, float(1 / np.sqrt(D)), _lib.VLLT_BF16, out.data_ptr(),
                                                 ws.data_ptr(), ws.numel(), _lib.stream_handle()))
    t = _event_times(torch, run, args.steps, args.warmup, dev)
    assert int(ws[:4].view(torch.int32).item()) == 0
    fl = 4.0 * D * H * S * P * (P + 1) / 2
    peak, kind = _tc_peak()
    if rank == 0:
        v = fl / t / 1e12
        print(json.dumps({"metric": "prefill attention TFLOP/s (causal, tcgen05)", "value": round(v, 1),
                          "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(t * 1e3, 4), "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1)",
                          "config": {"workload": f"{S} x {P}-token prompts, H{H}/KV{KV}/D{D}, block {bs}",
                                     "l2": "flushed before each launch"},
                          "roofline": {"bound": "tensor", "achieved": round(v, 1), "peak": peak, "unit": "TFLOP/s",
                                       "frac": round(v / peak, 3), "peak_kind": kind, "traffic": None}}),
              flush=True)


def main_decode(args, torch, dev, rank, world):
    s, t_step, t = decode_bench(torch, dev, args.steps, args.warmup)
    hbm, kind = peaks()
    if rank == 0:
        ach = s["attn_bytes"] / t / 1e9
        print(json.dumps({
            "metric": "paged-attention decode HBM GB/s", "value": round(ach, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_step * 1e3, 4),
            "attention_ms": round(t * 1e3, 4), "step_gbs": round(s["alg_bytes"] / t_step / 1e9, 1),
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1)",
            "config": {"workload": "C3 decode: 256 seqs, ctx U[1,4096], H32/KV8/D128, block 16",
                       "l2": "flushed before each step; KV > L2"},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 3), "traffic": None}}), flush=True)


def llama_config(num_blocks: int, max_seqs: int = 512, budget: int = 8192):
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    mc = ModelConfig(n_layers=32, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336, vocab_size=128256,
                     max_seq_len=9216, seed=0)
    return EngineConfig(model=mc,
                        cache=CacheConfig(block_size=16, num_blocks=num_blocks, enable_prefix_caching=False),
                        scheduler=SchedulerConfig(max_seqs=max_seqs, max_batched_tokens=budget))


def _progress(what: str) -> None:
    """One line on stderr per stage of a multi-rank run (where a stall happened)."""
    print(f"[rank {os.environ.get('RANK', '0')}] {what} {time.strftime('%H:%M:%S')}", file=sys.stderr, flush=True)


def allreduce_profile(torch, dev, comm, d_model, reps=20):
    """Device time (us, max over ranks) of one libvllt all-reduce
    (vllt_tp_allreduce_bf16: bf16, in place, the forward's collective after
    o_proj and down_proj) of `rows x d_model` for every token bucket the
    forward's graphs use. Every rank calls it with the same sizes, before the
    engine starts, so the ranks take the same collectives in the same order."""
    import torch.distributed as dist

    from vllt import _lib
    from vllt.runner import token_bucket

    L = _lib.lib()
    sizes = sorted({token_bucket(t) for t in range(1, 8193)})
    buf = torch.zeros(sizes[-1] * d_model, dtype=torch.bfloat16, device=dev)
    st = _lib.stream_handle()
    times = []
    for rows in sizes:
        n = rows * d_model
        for _ in range(3):
            _lib.check(L.vllt_tp_allreduce_bf16(buf.data_ptr(), n, comm, st))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            _lib.check(L.vllt_tp_allreduce_bf16(buf.data_ptr(), n, comm, st))
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / reps)
    t = torch.tensor(times, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return dict(zip(sizes, (round(float(x), 2) for x in t.cpu())))


def allreduce_share(pass_log, ar_us: dict, n_layers: int, max_tokens: int) -> float:
    """Seconds of all-reduce in the logged passes: two per layer, each of the
    pass's graph bucket (the rows the forward reduces)."""
    from vllt.runner import token_bucket

    return sum(2 * n_layers * ar_us[min(token_bucket(tokens), max_tokens)] for tokens, _, _, _ in pass_log) / 1e6


def main_llama(args, torch, dev, rank, world):
    """Llama-3-8B-shaped continuous batching, tensor parallel over all ranks:
    512 requests (prompt mean 1024, output mean 256), greedy, bf16."""
    from vllt.engine import gpu_engine
    from vllt.llama import LlamaRunner
    from vllt.tp import TPGroup, TPLlamaRunner
    from vllt.workloads import llama_workload

    cfg = llama_config(args.llama_blocks)
    group = TPGroup() if world > 1 else None
    ar_us = allreduce_profile(torch, dev, group.comm, cfg.model.d_model) if world > 1 else None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        hbm, tfl, kind = float(pk["hbm_gbs"]), float(pk["bf16_tflops_sustained"]), "measured (sustained bf16)"
    except Exception:
        hbm, tfl, kind = 6650.0, 1400.0, "fallback"
    if rank != 0:
        runner = TPLlamaRunner(cfg.model, cfg.cache, cfg.scheduler, group=group)
        _progress("worker ready")
        runner.worker_loop()
        _progress("worker stopped")
        t = torch.tensor([runner.marked_seconds()], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        runner.release_graphs()
        group.close()
        torch.distributed.destroy_process_group()
        return
    kw = dict(group=group) if world > 1 else {}
    eng = gpu_engine(cfg, runner_cls=TPLlamaRunner if world > 1 else LlamaRunner, **kw)
    run = eng.runner
    _progress("engine ready")
    for i in range(args.warmup):  # short requests: every graph bucket and kernel warmed
        run_workload(eng, llama_workload(16, seed=100 + i, out_mean=24), f"w{i}")
        _progress(f"warm-up {i} done")
    # as many short sequences as the timed run holds, with spread-out lengths: decode passes
    # shrink through every token bucket (graph) of the ladder before the timed region
    run_workload(eng, llama_workload(args.llama_requests, seed=99, prompt_mean=48, out_mean=40), "wd")
    _progress("decode warm-up done")
    reqs = llama_workload(args.llama_requests, seed=0)
    run.roofline_peaks = (hbm, tfl)
    run.roofline_s = 0.0
    run.pass_log = []
    flush_l2(torch, dev)
    torch.cuda.synchronize()
    l0 = run.L.vllt_kernel_launches() + run.replayed_kernels - run.captured_kernels
    if world > 1:
        run.mark(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t_wall = time.perf_counter()
    window = tuple(int(x) for x in args.nvtx_passes.split(":")) if args.nvtx_passes else None
    with Clocks(int(os.environ.get("LOCAL_RANK", 0))) as clk:
        toks, lat, steps = run_workload(eng, reqs, "t", window)
    e1.record()
    if world > 1:
        run.mark(1)
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    _progress("timed run done")
    elapsed = e0.elapsed_time(e1) / 1e3
    launches = run.L.vllt_kernel_launches() + run.replayed_kernels - run.captured_kernels - l0
    if world > 1:
        run.stop_workers()
        t = torch.tensor([run.marked_seconds()], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed = max(elapsed, float(t[0]))
    line = {
        "metric": f"engine output tok/s (Llama-3-8B shape, {len(reqs)} requests, tensor parallel {world})",
        "value": round(toks / elapsed, 1), "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": args.warmup,
        "ms_per_step": round(elapsed * 1e3, 1), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "impl": "vllt",
        "data": "synthetic (seeded N(0,0.02) weights, seeded lognormal requests)",
        "config": {"workload": "C4: 32L d4096 32/8 heads D128 ffn 14336 vocab 128256, 512 requests prompt mean 1024 "
                               "(32-8192) output mean 256 (16-1024), budget 8192, block 16, greedy",
                   "model": "Llama-3-8B shape (random init)", "global_batch": len(reqs), "seq_len": 9216,
                   "parallelism": f"tp{world}", "forward_passes": steps, "num_blocks": args.llama_blocks,
                   "warmup": f"{args.warmup} short 16-request workloads and one {args.llama_requests}-request "
                             "short workload (every decode bucket)", "l2": "flushed before the timed workload"},
        **latency_summary(lat, 1),
        "wall_s": round(t_wall, 3),
        "gpu_launches": int(launches),
        "e2e": None,
        "roofline": {"bound": "per forward pass max(HBM bytes / BW, FLOPs / bf16 peak), summed", "unit": "s",
                     "achieved": round(elapsed, 3), "peak": round(run.roofline_s, 3),
                     "frac": round(run.roofline_s / elapsed, 4), "peak_kind": kind, "hbm_gbs": hbm,
                     "bf16_tflops": tfl, "traffic": None},
        "clocks": clk.summary(),
    }
    ps = run.pass_summary()
    line["breakdown"] = dict(ps, host_and_other_s=round(elapsed - ps["gpu_s"], 3))
    if ar_us is not None:  # the tensor-parallel collectives' share of the forward passes
        ar_s = allreduce_share(run.pass_log, ar_us, cfg.model.n_layers, run.caps.max_tokens)
        line["breakdown"].update(allreduce_s_est=round(ar_s, 3),
                                 allreduce_share_of_pass_gpu=round(ar_s / max(ps["gpu_s"], 1e-9), 3),
                                 allreduce_us_by_rows={str(k): v for k, v in ar_us.items() if k in (16, 64, 256, 512, 1024, 8192)})
    print(json.dumps(line), flush=True)
    if world > 1:  # after the result line: graphs holding NCCL calls go before the communicators
        _progress("teardown")
        run.release_graphs()
        group.close()
        torch.distributed.destroy_process_group()
        _progress("done")


# ---- CPU baseline / reference arm ---------------------------------------------------------
def reference_run(workload: str, seed: int = 0):
    """The unmodified reference engine (NumpyRunner) on the same workload."""
    from vllmlite.engine import LLMEngine

    eng = LLMEngine(engine_config(workload))
    reqs = requests(workload, seed)
    t0 = time.perf_counter()
    toks, lat, steps = run_workload(eng, reqs, "r")
    return toks, time.perf_counter() - t0, lat, steps


def cpu_baseline(workload: str):
    try:
        import vllmlite  # noqa: F401
    except Exception as e:  # pragma: no cover
        return {"value": None, "unit": "tok/s", "unavailable": f"vllm-lite not importable: {e}"}
    reference_run(workload)  # warm-up (BLAS threads, page faults), as bench/bench.py:178-182
    best = None
    for _ in range(2):
        toks, t, lat, steps = reference_run(workload)
        if best is None or t < best[1]:
            best = (toks, t, lat)
    return {"value": round(best[0] / best[1], 1), "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
            "sample": f"whole 48-request {workload} workload, best of 2 after 1 warm-up, vllm-lite NumpyRunner "
                      f"(OpenBLAS threads={os.environ.get('OPENBLAS_NUM_THREADS', 'all')})",
            **latency_summary(best[2])}


def main_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    try:
        import vllmlite  # noqa: F401
    except Exception as e:
        print(json.dumps({"impl": "reference", "unavailable": f"vllm-lite not importable: {e}"}))
        return
    if args.workload not in ("mixed", "shared", "decode"):
        why = {"llama8b": "the reference runs the Llama-3-8B shape only in NumPy on the host, impractical at "
                          "this size (a 2-layer slice is its CPU parity check)",
               "spec": "run the reference's speculative engine through --workload spec's own cpu_baseline",
               "gemm": "the reference has no separate projection kernels (NumPy matmul inside its forward)",
               "prefill": "the reference has no separate prefill attention (NumPy inside its forward)"}
        print(json.dumps({"impl": "reference", "unavailable": why[args.workload]}), flush=True)
        return
    wl = "mixed" if args.workload == "decode" else args.workload
    for _ in range(args.warmup):
        reference_run(wl)
    toks = t = 0.0
    lats = []
    for _ in range(args.steps):
        n, dt, lat, steps = reference_run(wl)
        toks += n
        t += dt
        lats.append(lat)
    v = round(toks / t, 1)
    print(json.dumps({
        "metric": "engine output tok/s (48-request mixed-length greedy workload)" if wl == "mixed"
        else "engine output tok/s (48-request shared-prefix workload, prefix cache on)",
        "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * t / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(v / PUBLISHED[wl], 3), "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"C1 {wl}", "model": "TinyLlama-style 6L/384d", "global_batch": 48,
                   "seq_len": 768 if wl == "shared" else 512, "parallelism": "none (host CPU)"},
        **latency_summary(merge_latency(lats)),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                         "sample": f"{args.steps} whole workloads, vllm-lite NumpyRunner"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="mixed", choices=["mixed", "shared", "decode", "llama8b", "spec", "gemm",
                                                               "prefill"])
    ap.add_argument("--spec-k", type=int, default=4)
    ap.add_argument("--gemm-m", default="", help="token counts of the gemm workload (default 8192,512,256,64)")
    ap.add_argument("--gemm-shape", default="", help="projections of the gemm workload (qkv,o_proj,gate_up,down)")
    ap.add_argument("--nvtx-passes", default="", help="a:b - mark engine steps a..b-1 of the (first) timed run "
                                                      "with an NVTX range (profiling)")
    ap.add_argument("--llama-requests", type=int, default=512)
    ap.add_argument("--llama-blocks", type=int, default=45000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        main_reference(args)
    else:
        main_ours(args)


if __name__ == "__main__":
    main()
