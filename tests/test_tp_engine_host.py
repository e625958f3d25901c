"""CPU, two gloo ranks: the tensor-parallel serving path, TPLlamaRunner's own
protocol code over the host build of libvllt.

tests/host_runner.py HostTPRunner keeps TPLlamaRunner's launch (the record
broadcast, the copy-on-write message), vocab-parallel greedy_picks,
gather_rows and stop, and runs the shard forward of the host build with its
all-reduce handed to gloo; rank 1 serves TPLlamaRunner's worker protocol
(vllt.tp.serve). Rank 0 runs the same requests twice on a narrow Llama-shaped
model:
  * the reference's unmodified LLMEngine, whose host sample() reads the
    full-vocabulary logits gathered from both ranks' slices;
  * vllt's GpuLLMEngine with run-ahead: greedy rows merged from both ranks'
    (max, index) pairs, rows with a min_tokens EOS mask, a repetition penalty
    or a temperature draw gathered whole and picked by the device kernels,
    passes launched before the previous pass's tokens reached the host (the
    worker keeps the merged picks for the stand-ins).
Both engines see the same logits every pass, so their token streams must be
equal, with passes run ahead in the second and every worker message served.
"""

import datetime
import json
import os
import socket
import sys

import numpy as np
import pytest

from tests.conftest import needs_vllmlite

torch = pytest.importorskip("torch")
pytestmark = needs_vllmlite

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODES = ("reference", "gpu")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config():
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    mc = ModelConfig(n_layers=2, n_heads=4, n_kv_heads=2, d_model=512, d_ff=512, vocab_size=300, max_seq_len=512,
                     seed=3)
    return EngineConfig(model=mc, cache=CacheConfig(block_size=16, num_blocks=64),
                        scheduler=SchedulerConfig(max_seqs=4, max_batched_tokens=64))


def _requests():
    from vllmlite.sequence import SamplingParams

    rng = np.random.default_rng(7)
    toks = [[int(t) for t in rng.integers(1, 300, size=n)] for n in (30, 90, 9, 50, 20)]
    params = [SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True),
              SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True),
              SamplingParams(max_tokens=8, temperature=0.7, top_k=40, top_p=0.9, seed=5, ignore_eos=True),
              SamplingParams(max_tokens=8, temperature=0.0, repetition_penalty=1.3, ignore_eos=True),
              SamplingParams(max_tokens=8, temperature=0.0, min_tokens=6)]
    return toks, params


def _rank(rank, world, port, lib_path, result_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-lite_b200"), os.path.join(ROOT, "baseline", "_ref")]
    import ctypes as C
    from types import SimpleNamespace

    import torch.distributed as dist

    import vllt._lib as _lib
    from tests.host_build import load_library_host
    from tests.host_runner import HostTPRunner
    from vllt.engine import GpuLLMEngine, cuda_engine

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        L = load_library_host(lib_path)
        _lib._lib, _lib.stream_handle = L, (lambda stream=None: 0)
        AllReduce = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int64, C.c_void_p)

        def allreduce(buf, count, comm):
            if comm != HostTPRunner.COMM:
                return 1
            dist.all_reduce(torch.frombuffer((C.c_uint16 * count).from_address(buf), dtype=torch.bfloat16))
            return 0

        hook = AllReduce(allreduce)
        L.vllt_host_set_allreduce.argtypes = [AllReduce]
        L.vllt_host_set_allreduce(hook)
        HostTPRunner.lib, HostTPRunner.group = L, SimpleNamespace(rank=rank, world=world)
        cfg = _config()
        res = {}
        for mode in MODES:  # every rank builds one runner per engine, in the same order
            if rank == 0:
                kw = dict(engine_cls=GpuLLMEngine.resolve()) if mode == "gpu" else {}
                eng = cuda_engine(cfg, runner_cls=HostTPRunner, **kw)
                toks, params = _requests()
                ids = [eng.add_request(params=p, prompt_token_ids=t) for t, p in zip(toks, params)]
                while eng.has_work:
                    eng.step()
                res[mode] = dict(streams=[eng.seqs[i].output_token_ids for i in ids],
                                 ahead=getattr(eng, "passes_ahead", 0), steps=eng.runner.steps)
                eng.runner.stop_workers()
            else:
                run = HostTPRunner(cfg.model, cfg.cache, cfg.scheduler)
                res[mode] = dict(passes=run.worker_loop())
        L.vllt_host_set_allreduce(AllReduce())
        with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_engine_serves_the_reference_engines_streams(host_library, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _free_port(), host_library._name, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0, r1 = (json.load(open(tmp_path / f"rank{r}.json")) for r in range(2))
    ref, gpu = r0["reference"], r0["gpu"]
    assert gpu["streams"] == ref["streams"]
    assert [len(s) for s in ref["streams"]] == [8] * 5
    assert gpu["ahead"] > 0
    for mode in MODES:  # the worker served every pass rank 0 ran
        assert r1[mode]["passes"] == r0[mode]["steps"] > 0
