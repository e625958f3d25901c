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
  * an oversize record is refused on rank 0 before anything is broadcast.
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

    from vllt.tp import (CTRL_WORDS, OP_FORWARD, OP_GATHER, OP_MARK, OP_STOP, ControlPlane, gather_vocab_rows,
                         merge_argmax, serve)

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
                plane.send(OP_FORWARD, rec, b, g)
                if j == 2:
                    plane.send(OP_GATHER, GATHER_ROWS)
            plane.send(OP_MARK)
            plane.send(OP_STOP)
        else:
            seen, marks, gathers = [], [], []

            def forward(bounds, greedy):
                n = int(plane.ctrl[7])
                seen.append((plane.buf[:n].numpy().copy(), bounds, greedy))

            def gather(n):
                gathers.append((len(seen), plane.buf[:n].numpy().copy()))

            assert serve(plane, forward, marks.append, gather) == len(msgs)
            assert marks == [0, 0]
            for (rec, b, g), (got, gb, gg) in zip(msgs, seen):
                np.testing.assert_array_equal(got, rec)
                assert [getattr(gb, f) for f in FIELDS] == [getattr(b, f) for f in FIELDS] and gg == g
            assert len(gathers) == 1 and gathers[0][0] == 3
            np.testing.assert_array_equal(gathers[0][1], GATHER_ROWS)

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
