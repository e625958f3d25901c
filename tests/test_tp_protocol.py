"""CPU, two gloo ranks: the tensor-parallel host protocol.

The GPU path (vllt.tp.TPLlamaRunner) broadcasts one int32 message per forward
pass (step record + control words) and merges per-rank (max, index) pairs for
vocab-parallel greedy. Both pieces run here exactly as the GPU path uses them,
over gloo with CPU tensors and a recording stand-in for the forward:
  * every message rank 0 sends arrives intact and in order, records of
    different lengths included, with marks interleaved, and the stop message
    ends the worker loop with the right pass count;
  * the merged argmax equals np.argmax over the full (unsharded) logits,
    with planted ties inside a slice and across the slice boundary;
  * a gather message (rows that need the whole vocabulary for their pick:
    EOS mask, repetition penalty, temperature draw) reaches the worker's
    gather handler with its row list, and the all-gather of every rank's
    slice of those rows rebuilds the full rows in vocabulary order;
  * an oversize record is refused on rank 0 before anything is broadcast;
  * run-ahead: rank 0's engine launches a pass before it has read the
    previous pass's picks, with stand-in tokens in the record, and the worker
    resolves them from its own copy of the merged greedy picks exactly as
    rank 0 does. Streams and the step count equal the reference engine's,
    and passes with rows picked on rank 0 only do not run ahead.
"""

import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIELDS = ("tokens", "rows", "decode_seqs", "tiles", "max_ctx")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _messages():
    from vllt._lib import StepBounds

    rng = np.random.default_rng(5)
    out = []
    for i in range(6):
        n = int(rng.integers(4, 60))
        rec = rng.integers(-5, 1 << 20, size=n).astype(np.int32)
        b = StepBounds(*[int(x) for x in rng.integers(1, 5000, size=5)])
        out.append((rec, b, i % 2))
    return out


GATHER_ROWS = np.asarray([5, 0, 3], np.int32)
COW_PAIRS = np.asarray([7, 12, 3, 40], np.int32)  # (src, dst) block pairs, flat


def _logits(R, V):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((R, V)).astype(np.float32)
    half = V // 2
    x[0, 3] = x[0, half + 1] = 50.0          # tie across the two slices -> rank 0's index
    x[1, half + 2] = x[1, half + 7] = 60.0   # tie inside rank 1's slice -> the first
    x[2, 5] = x[2, 6] = 70.0                 # tie inside rank 0's slice
    x[3, :] = 1.0                            # every entry equal -> index 0
    return x


def _rank(rank, world, port, result_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-lite_b200")]
    import torch.distributed as dist

    from vllt.tp import (CTRL_WORDS, OP_COW, OP_FORWARD, OP_GATHER, OP_MARK, OP_STOP, ControlPlane,
                         gather_vocab_rows, merge_argmax, serve)

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plane = ControlPlane(torch.zeros(64 + CTRL_WORDS, dtype=torch.int32))
        msgs = _messages()
        if rank == 0:
            with pytest.raises(ValueError):
                plane.send(OP_FORWARD, np.zeros(65, np.int32))
            plane.send(OP_MARK)
            for j, (rec, b, g) in enumerate(msgs):
                if j == 4:  # a pass with copy-on-write pairs: the copy message goes first
                    plane.send(OP_COW, COW_PAIRS)
                plane.send(OP_FORWARD, rec, b, g)
                if j == 2:
                    plane.send(OP_GATHER, GATHER_ROWS)
            plane.send(OP_MARK)
            plane.send(OP_STOP)
        else:
            seen, marks, gathers, cows = [], [], [], []

            def forward(bounds, greedy):
                n = int(plane.ctrl[7])
                seen.append((plane.buf[:n].numpy().copy(), bounds, greedy))

            def gather(n):
                gathers.append((len(seen), plane.buf[:n].numpy().copy()))

            def cow(n):
                cows.append((len(seen), plane.buf[:n].numpy().copy()))

            assert serve(plane, forward, marks.append, gather, cow) == len(msgs)
            assert marks == [0, 0]
            for (rec, b, g), (got, gb, gg) in zip(msgs, seen):
                np.testing.assert_array_equal(got, rec)
                assert [getattr(gb, f) for f in FIELDS] == [getattr(b, f) for f in FIELDS] and gg == g
            assert len(gathers) == 1 and gathers[0][0] == 3
            np.testing.assert_array_equal(gathers[0][1], GATHER_ROWS)
            assert len(cows) == 1 and cows[0][0] == 4  # before the pass it belongs to
            np.testing.assert_array_equal(cows[0][1], COW_PAIRS)

        # vocab-parallel greedy: rank r owns columns [r*V/2, (r+1)*V/2)
        R, V = 8, 40
        x = _logits(R, V)
        vl = V // world
        sl = x[:, rank * vl:(rank + 1) * vl]
        val = torch.from_numpy(sl.max(1))
        idx = torch.from_numpy((sl.argmax(1) + rank * vl).astype(np.int32))
        vals = torch.empty(world * R, dtype=torch.float32)
        idxs = torch.empty(world * R, dtype=torch.int32)
        dist.all_gather(list(vals.view(world, R)), val)
        dist.all_gather(list(idxs.view(world, R)), idx)
        got = merge_argmax(vals.view(world, R), idxs.view(world, R)).numpy()
        np.testing.assert_array_equal(got, x.argmax(1))
        # full rows of the gathered logit rows, from every rank's slice
        full = gather_vocab_rows(torch.from_numpy(sl[GATHER_ROWS]), world).numpy()
        np.testing.assert_array_equal(full, x[GATHER_ROWS])
        open(os.path.join(result_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_control_plane_and_vocab_parallel_greedy_over_gloo(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]


def _silent_peer(rank, world, port, result_dir, who_stops):
    """One rank stops taking part in the protocol; the other must get an error
    from its next collective within the process group's timeout (2 s), not
    hang. who_stops = 0: rank 0 sends one forward message, then nothing (a
    driver that died or hung); the worker's receive fails. who_stops = 1: the
    worker takes one message, then never joins another collective; rank 0's
    vocab-parallel all-gather after its next forward fails."""
    import datetime
    import time

    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-lite_b200")]
    import torch.distributed as dist

    from vllt.tp import CTRL_WORDS, OP_FORWARD, ControlPlane, serve

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=2))
    plane = ControlPlane(torch.zeros(16 + CTRL_WORDS, dtype=torch.int32))
    rec = np.arange(5, dtype=np.int32)
    result = "none"
    if rank == who_stops:
        if rank == 0:
            plane.send(OP_FORWARD, rec)
        else:
            plane.recv()
        time.sleep(6)  # alive but silent: never joins another collective
        result = "silent"
    else:
        t0 = time.monotonic()
        try:
            if rank == 0:
                plane.send(OP_FORWARD, rec)  # the worker took this one
                plane.send(OP_FORWARD, rec)  # a broadcast only sends: it may complete
                vals = torch.empty(2 * 4)
                dist.all_gather(list(vals.view(2, 4)), torch.zeros(4))  # needs the worker's slice
            else:
                serve(plane, lambda b, g: None, lambda t: None)
            result = "no error"
        except RuntimeError as e:
            dt = time.monotonic() - t0
            result = f"error {dt:.1f}" if dt < 5.0 else f"late error {dt:.1f}"
            print(f"rank {rank} ({type(e).__name__}): {str(e)[:120]}", flush=True)
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write(result)
    os._exit(0)  # the group cannot be torn down collectively with a silent peer


@pytest.mark.parametrize("who_stops", [0, 1])
def test_a_silent_rank_turns_into_an_error_within_the_timeout(tmp_path, who_stops):
    import torch.multiprocessing as mp

    mp.start_processes(_silent_peer, args=(2, _free_port(), str(tmp_path), who_stops), nprocs=2, join=True,
                       start_method="spawn")
    got = {f: open(os.path.join(tmp_path, f)).read() for f in os.listdir(tmp_path)}
    waiting = f"rank{1 - who_stops}"
    assert got[f"rank{who_stops}"] == "silent"
    assert got[waiting].startswith("error "), got


# ---- run-ahead under tensor parallelism -------------------------------------------
# Rank 0 runs GpuLLMEngine (run-ahead on) over TwoRankRunner, which speaks the
# real protocol (ControlPlane messages, vocab-parallel greedy through
# merge_argmax, gather messages for rows that need the whole vocabulary); the
# forward is the reference NumpyRunner on rank 0, whose logits travel to the
# worker in a test-only broadcast after each forward message. Each rank
# builds the pass's metadata with the builder's host-compiled code against its
# own pick buffer; the worker checks its resolved tokens equal rank 0's,
# which rank 0 checks against the true tokens.


def _ahead_requests():
    from vllmlite.sequence import SamplingParams

    from vllt.workloads import mixed_workload

    reqs = mixed_workload(8, 4, 0)
    for _, _, p in reqs:
        p.max_tokens = min(p.max_tokens, 24)
    ids = reqs[0][1]
    # rows picked on rank 0 only: a repetition penalty and a seeded temperature draw
    reqs.append(("pen", ids[:40], SamplingParams(max_tokens=10, temperature=0.0, repetition_penalty=1.3,
                                                 ignore_eos=True)))
    reqs.append(("tmp", ids[:30], SamplingParams(max_tokens=10, temperature=0.8, top_k=20, seed=3, ignore_eos=True)))
    return reqs


def _ahead_config():
    from vllmlite.config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig

    from tests import fixtures as F

    return EngineConfig(model=ModelConfig(vocab_size=261, **F.TINY),
                        cache=CacheConfig(block_size=16, num_blocks=512),
                        scheduler=SchedulerConfig(max_seqs=8, max_batched_tokens=64))


class _Meta:
    """The metadata builder compiled for the host, resolving record tokens."""

    def __init__(self, so_path, cfg):
        import ctypes

        from vllt import _lib
        from vllt.runner import tile_positions

        self.lib = ctypes.CDLL(so_path)
        self.lib.build_meta_host.argtypes = ([ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 8 +
                                             [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int])
        self.caps = _lib.Caps(64, 2048, 256, 64)
        self.pool = np.full((128, self.caps.max_table_width), -1, np.int32)
        self.bs, self.nb, self.vocab = cfg.cache.block_size, cfg.cache.num_blocks, cfg.model.vocab_size
        self.qp = tile_positions(cfg.model.n_heads // cfg.model.n_kv_heads)

    def tokens(self, rec, picks):
        import ctypes

        from vllt import _lib

        L = _lib.lib()
        meta = np.zeros(L.vllt_meta_bytes(ctypes.byref(self.caps)) // 4, np.int32)
        rec = np.ascontiguousarray(rec, np.int32)
        c = self.caps
        err = self.lib.build_meta_host(rec.ctypes.data, self.pool.ctypes.data, self.pool.shape[0], c.max_seqs,
                                       c.max_tokens, c.max_rows, c.max_table_width, self.bs, self.nb, self.qp,
                                       meta.ctypes.data, picks.ctypes.data, picks.size, self.vocab)
        assert err == 0
        off = (L.vllt_meta_field(ctypes.c_void_p(meta.ctypes.data), ctypes.byref(c), 8) - meta.ctypes.data) // 4
        return meta[off:off + int(rec[1])].copy()


def _vocab_slice(full, rank):
    """Rank's half of the vocabulary (the logits padded to an even width with
    -inf, as the real runner's vocabulary divides evenly by the ranks)."""
    V = full.shape[1]
    h = (V + 1) // 2
    pad = np.full((full.shape[0], 2 * h), -np.inf, np.float32)
    pad[:, :V] = full
    return pad[:, rank * h:(rank + 1) * h]


def _local_greedy(logits_slice, rank, world, R):
    import torch.distributed as dist

    from vllt.tp import merge_argmax

    vl = logits_slice.shape[1]
    val = torch.from_numpy(logits_slice[:R].max(1).astype(np.float32))
    idx = torch.from_numpy((logits_slice[:R].argmax(1) + rank * vl).astype(np.int32))
    vals = torch.empty(world * R, dtype=torch.float32)
    idxs = torch.empty(world * R, dtype=torch.int32)
    dist.all_gather(list(vals.view(world, R)), val)
    dist.all_gather(list(idxs.view(world, R)), idx)
    return merge_argmax(vals.view(world, R), idxs.view(world, R))


def _payload(tokens=None, logits=None):
    """Test-only broadcast after a forward message: rank 0's resolved tokens
    and the pass's full logits (sizes first)."""
    import torch.distributed as dist

    sizes = torch.zeros(3, dtype=torch.int64)
    if tokens is not None:
        sizes[:] = torch.tensor([tokens.size, logits.shape[0], logits.shape[1]])
    dist.broadcast(sizes, src=0)
    T, R, V = (int(x) for x in sizes)
    buf = torch.zeros(T + R * V, dtype=torch.float32)
    if tokens is not None:
        buf[:T] = torch.from_numpy(tokens.astype(np.float32))
        buf[T:] = torch.from_numpy(logits.reshape(-1))
    dist.broadcast(buf, src=0)
    return buf[:T].numpy().astype(np.int64), buf[T:].numpy().reshape(R, V)


class TwoRankRunner:
    """Rank 0's runner: the tensor-parallel runner's interface over gloo."""

    tp_size = 2

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, device=None, lib=None, plane=None, meta=None):
        from types import SimpleNamespace

        from vllmlite.runner import NumpyRunner

        from vllt.runner import CudaRunner, StepPacker

        self.check_step_flags = CudaRunner.check_step_flags.__get__(self)
        self.ref = NumpyRunner(model_cfg, cache_cfg)
        self.model_cfg, self.L, self.plane, self.mt = model_cfg, lib, plane, meta
        self.dev = torch.device("cpu")
        self.meta = torch.zeros(16, dtype=torch.int32)
        self.w = SimpleNamespace(vocab_padded=model_cfg.vocab_size)
        self.picks_dev = torch.zeros(1024, dtype=torch.int32)
        self.packer = StepPacker(meta.bs, meta.nb, model_cfg.vocab_size, model_cfg.max_seq_len, meta.qp,
                                 pool_slots=128, pool_width=meta.caps.max_table_width, token_refs=1024)
        self.stand_ins = 0

    def pick_buffer(self, n):
        return self.picks_dev[:n]

    def launch(self, out):
        from vllt.runner import _tokens
        from vllt.tp import OP_FORWARD

        rec, bounds, rows, (S, T, R, W) = self.packer.pack(out)
        picks = self.picks_dev.numpy()
        tokens = self.mt.tokens(rec, picks)
        saved = []
        for item in out.scheduled:
            o = item.seq.output_token_ids
            for k, t in enumerate(o):
                if t < 0:
                    saved.append((o, k, t))
                    o[k] = int(picks[-t - 1])
        self.stand_ins += len(saved)
        try:
            want = [t for item in out.scheduled for t in _tokens(item.seq, item.start_pos, item.num_tokens)]
            assert tokens.tolist() == want
            logits, _ = self.ref.execute(out)
        finally:
            for o, k, t in saved:
                o[k] = t
        self.plane.send(OP_FORWARD, rec, bounds, greedy=1)
        _payload(tokens, logits.astype(np.float32))
        self.full = logits.astype(np.float32)
        self.logits_dev = torch.from_numpy(self.full)
        return rows, R

    def greedy_picks(self, R):
        return _local_greedy(_vocab_slice(self.full, 0), 0, 2, R)

    def gather_rows(self, rows):
        from vllt.tp import OP_GATHER, gather_vocab_rows

        rows = np.asarray(rows, np.int32)
        self.plane.send(OP_GATHER, rows)
        V = self.full.shape[1]
        full = gather_vocab_rows(torch.from_numpy(np.ascontiguousarray(_vocab_slice(self.full, 0)[rows])), 2)
        return full[:, :V].contiguous()


def _ahead_rank(rank, world, port, result_dir, so_path):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "vllm-lite_b200"), os.path.join(ROOT, "baseline", "_ref")]
    import torch.distributed as dist

    import vllt._lib as _lib
    from vllt.tp import CTRL_WORDS, OP_STOP, ControlPlane, gather_vocab_rows, serve

    _lib.stream_handle = lambda stream=None: 0
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _ahead_config()
        meta = _Meta(so_path, cfg)
        plane = ControlPlane(torch.zeros(4096 + CTRL_WORDS, dtype=torch.int32))
        if rank == 0:
            from vllmlite.engine import LLMEngine

            from tests.test_engine_host import OracleLib
            from vllt.engine import GpuLLMEngine, cuda_engine

            reqs = _ahead_requests()
            ref = LLMEngine(_ahead_config())
            ids = [ref.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
            while ref.has_work:
                ref.step()
            want = [ref.seqs[i].output_token_ids for i in ids]
            reqs = _ahead_requests()
            eng = cuda_engine(cfg, engine_cls=GpuLLMEngine.resolve(), runner_cls=TwoRankRunner, lib=OracleLib(),
                              plane=plane, meta=meta)
            ids = [eng.add_request(params=p, request_id=r, prompt_token_ids=t) for r, t, p in reqs]
            while eng.has_work:
                eng.step()
            plane.send(OP_STOP)
            got = [eng.seqs[i].output_token_ids for i in ids]
            assert got == want and eng.total_steps == ref.total_steps
            assert 0 < eng.passes_ahead < eng.total_steps and eng.runner.stand_ins > 0
        else:
            picks = np.zeros(1024, np.int32)
            last = {}

            def forward(bounds, greedy):
                tokens = meta.tokens(plane.buf[:int(plane.ctrl[7])].numpy(), picks)
                want_tokens, full = _payload()
                assert tokens.tolist() == want_tokens.tolist()  # stand-ins resolve as on rank 0
                last["full"] = full
                if greedy:
                    picks[:bounds.rows] = _local_greedy(_vocab_slice(full, 1), 1, 2, bounds.rows).numpy()

            def gather(n):
                rows = plane.buf[:n].numpy().copy()
                gather_vocab_rows(torch.from_numpy(np.ascontiguousarray(_vocab_slice(last["full"], 1)[rows])), 2)

            assert serve(plane, forward, lambda tag: None, gather) > 0
        open(os.path.join(result_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_run_ahead_over_two_ranks(tmp_path):
    """Tensor-parallel run-ahead, two gloo ranks: the engine's streams and
    step count equal the reference engine's, passes with only plain greedy
    picks run ahead while the penalised / sampled ones (picked on rank 0
    after a gather) do not, and every record's stand-ins resolve on the worker
    exactly as on rank 0."""
    import torch.multiprocessing as mp

    from tests.conftest import have_vllmlite
    from tests.host_build import build_harness

    if not have_vllmlite():
        pytest.skip("vllm-lite (the host engine) is not importable")
    path = build_harness("meta_host", str(tmp_path), load=False)
    if path is None:
        pytest.skip("g++ is not available")
    out = tmp_path / "out"
    out.mkdir()
    mp.start_processes(_ahead_rank, args=(2, _free_port(), str(out), path), nprocs=2, join=True,
                       start_method="spawn")
    assert sorted(os.listdir(out)) == ["ok0", "ok1"]
