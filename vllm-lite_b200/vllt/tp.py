"""Tensor parallelism for the Llama-shaped bf16 model (one process per GPU).

Rank 0 runs the reference engine (Scheduler, BlockManager, sampling rules and
proposer, unchanged) with `TPLlamaRunner`; ranks > 0 run `worker_loop`. Per
forward pass:
  1. rank 0 packs the step record (same format as the 1-GPU runner) plus a
     control block and broadcasts it (torch.distributed, NCCL);
  2. every rank runs its shard: column-parallel QKV / gate-up, row-parallel
     o_proj / down_proj with a bf16 NCCL all-reduce inside libvllt's forward;
     every rank holds the same block ids for its own KV heads;
  3. greedy picks are vocab-parallel: each rank reduces its vocabulary slice to
     (max, first index) per row, the pairs are all-gathered and the lowest
     global index among the maxima wins (np.argmax semantics); every rank
     keeps the merged picks in its pick buffer, so a record that refers to
     them (rank 0's engine running ahead) resolves the same on every rank;
  4. a pass with copy-on-write pairs (a shared, partly filled block the
     scheduler forks: block_manager.py:77-93) is preceded by one copy
     message carrying the pairs; every rank copies the blocks of its own KV
     heads before the forward (runner.py:63-64 applies them first too);
  5. rows whose pick needs the whole vocabulary at once (a min_tokens EOS mask,
     a repetition penalty, or a temperature draw: sampling.py:41-64) are named
     in a gather message; every rank contributes its slice of those rows and
     rank 0 runs the single-GPU sampling kernels on the full rows.
All ranks take the same collective steps in the same order; a stop record ends
the workers.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import StepBounds, check, lib
from .llama import LlamaRunner
from .runner import CudaRunner

OP_FORWARD, OP_STOP, OP_MARK, OP_GATHER, OP_COW = 1, 2, 3, 4, 5
CTRL_WORDS = 8  # [op, tokens, rows, decode_seqs, tiles, max_ctx, greedy, record words]


class TPGroup:
    """libvllt's NCCL communicator for this process's rank (torch.distributed
    must already be initialised with one process per GPU)."""

    def __init__(self):
        import torch
        import torch.distributed as dist

        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        dev = torch.device("cuda", torch.cuda.current_device())
        uid = (C.c_uint8 * 128)()
        if self.rank == 0:
            check(lib().vllt_tp_unique_id(uid))
        t = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device=dev)
        dist.broadcast(t, src=0)
        uid = (C.c_uint8 * 128)(*t.cpu().tolist())
        comm = C.c_void_p()
        check(lib().vllt_tp_init(uid, self.rank, self.world, C.byref(comm)))
        self.comm = comm.value

    def close(self):
        if self.comm:
            check(lib().vllt_tp_destroy(self.comm))
            self.comm = None


class ControlPlane:
    """The per-pass message from rank 0 to the other ranks: the step record
    followed by CTRL_WORDS control words, in one int32 buffer that is broadcast
    whole, so every rank takes exactly one collective per message.

    `buf` is the broadcast buffer (on the GPU for NCCL, on the CPU for gloo);
    `host` is rank 0's staging copy (pinned memory on a GPU; omitted when `buf`
    is already host memory)."""

    def __init__(self, buf, host=None):
        import torch

        self.buf = buf
        self.host = buf if host is None else host
        self.capacity = buf.numel() - CTRL_WORDS
        self.ctrl = torch.zeros(CTRL_WORDS, dtype=torch.int32)
        self._staged = None  # CUDA event after the last host->device copy out of `host`

    def send(self, op: int, rec=None, bounds=None, greedy: int = 0) -> int:
        """Rank 0: broadcast one message; returns the bytes staged host->device."""
        import torch
        import torch.distributed as dist

        n = 0 if rec is None else int(rec.size)
        if n > self.capacity:
            raise ValueError(f"step record of {n} words exceeds the broadcast buffer ({self.capacity})")
        if self._staged is not None:
            # the previous message's copy out of the pinned staging buffer is
            # asynchronous: let it finish before the buffer is overwritten
            self._staged.synchronize()
            self._staged = None
        if n:
            self.host[:n].numpy()[:] = rec
        b = bounds or StepBounds(0, 0, 0, 0, 1)
        self.host[-CTRL_WORDS:].numpy()[:] = [op, b.tokens, b.rows, b.decode_seqs, b.tiles, b.max_ctx, greedy, n]
        staged = 0
        if self.host is not self.buf:
            if n:
                self.buf[:n].copy_(self.host[:n], non_blocking=True)
            self.buf[-CTRL_WORDS:].copy_(self.host[-CTRL_WORDS:], non_blocking=True)
            staged = 4 * (n + CTRL_WORDS)
            if self.buf.is_cuda:
                self._staged = torch.cuda.Event()
                self._staged.record()
        dist.broadcast(self.buf, src=0)
        return staged

    def recv(self):
        """Ranks > 0: take one message; returns (op, bounds, greedy, record words).
        The record itself stays in `buf[:n]` where the forward reads it."""
        import torch.distributed as dist

        dist.broadcast(self.buf, src=0)
        self.ctrl.copy_(self.buf[-CTRL_WORDS:])
        c = [int(x) for x in self.ctrl.tolist()]
        return c[0], StepBounds(*c[1:6]), c[6], c[7]


def serve(plane: ControlPlane, forward, mark, gather=None, cow=None) -> int:
    """Worker dispatch loop: forward(bounds, greedy) for each OP_FORWARD,
    mark(tag) for each OP_MARK, gather(n) for each OP_GATHER (the n row
    indices sit in the broadcast buffer), cow(n) for each OP_COW (n / 2
    (src, dst) block pairs in the buffer), return the number of passes at
    OP_STOP. An unknown op is a protocol error (rank 0 never sends one)."""
    passes = 0
    while True:
        op, bounds, greedy, n = plane.recv()
        if op == OP_STOP:
            return passes
        if op == OP_MARK:
            mark(bounds.tokens)
        elif op == OP_FORWARD:
            forward(bounds, greedy)
            passes += 1
        elif op == OP_GATHER and gather is not None:
            gather(n)
        elif op == OP_COW and cow is not None:
            cow(n)
        else:
            raise RuntimeError(f"tensor-parallel control: unknown op {op}")


def gather_vocab_rows(local, world: int):
    """Every rank's vocabulary slice of the same rows -> the full rows.
    local: [n, V/world] on this rank; returns [n, V] with rank r's slice at
    columns [r*V/world, (r+1)*V/world) (the lm_head row split of vllt.llama),
    identical on every rank. One all-gather."""
    import torch
    import torch.distributed as dist

    n, vl = local.shape
    parts = torch.empty((world * n, vl), dtype=local.dtype, device=local.device)  # rank-major
    dist.all_gather_into_tensor(parts, local.contiguous())
    return parts.view(world, n, vl).permute(1, 0, 2).reshape(n, world * vl).contiguous()


def merge_argmax(vals, idxs):
    """Vocab-parallel greedy: vals/idxs [ranks][R] hold each rank's (max logit,
    global index of its first maximum) per row, rank r owning the r-th
    vocabulary slice. Returns the global argmax per row with np.argmax's tie
    rule: among equal maxima the lowest index, i.e. the lowest rank."""
    import torch

    n = vals.shape[0]
    best = vals.max(0).values
    score = torch.where(vals == best, torch.arange(n, 0, -1, device=vals.device).view(n, 1), 0)
    return idxs.gather(0, score.argmax(0, keepdim=True)).view(-1)


class TPLlamaRunner(LlamaRunner):
    """One tensor-parallel shard; on rank 0 it is the engine's runner."""

    def __init__(self, model_cfg, cache_cfg, sched_cfg=None, *, group: TPGroup, max_rows: int | None = None, **kw):
        self.group = group
        super().__init__(model_cfg, cache_cfg, sched_cfg, tp_rank=group.rank, tp_size=group.world,
                         tp_comm=group.comm, **kw)
        # fixed capacities on every rank: the record buffer has one size everywhere
        c = self.caps
        self._reserve(c.max_seqs, c.max_tokens, max_rows or c.max_rows, c.max_table_width)
        self._fixed = True
        import torch

        self.plane = ControlPlane(self.rec_dev, self.rec_host)
        self._val = torch.empty(self.caps.max_rows, dtype=torch.float32, device=self.dev)
        self._idx = torch.empty(self.caps.max_rows, dtype=torch.int32, device=self.dev)
        self._vals = torch.empty(group.world * self.caps.max_rows, dtype=torch.float32, device=self.dev)
        self._idxs = torch.empty(group.world * self.caps.max_rows, dtype=torch.int32, device=self.dev)
        self._pending_rows = 0

    def _reserve(self, S, T, R, W):
        if getattr(self, "_fixed", False):
            c = self.caps
            if S > c.max_seqs or T > c.max_tokens or R > c.max_rows or W > c.max_table_width:
                raise ValueError(f"step exceeds the tensor-parallel capacities {(c.max_seqs, c.max_tokens, c.max_rows, c.max_table_width)}")
            return
        super()._reserve(S, T, R, W)
        import torch

        # the control block lives in the last CTRL_WORDS words of the record buffer
        extra = torch.empty(self.rec_dev.numel() + CTRL_WORDS, dtype=torch.int32, device=self.dev)
        self.rec_dev = extra
        self.rec_host = torch.empty(extra.numel(), dtype=torch.int32, pin_memory=True)

    # ---- rank 0 -------------------------------------------------------------------
    def launch(self, out):  # replaces LlamaRunner.launch (which is CudaRunner's plus the roofline)
        if out.cow:  # every rank forks the blocks of its KV heads before the forward
            pairs = np.asarray(out.cow, np.int64).reshape(-1, 2)
            if int(pairs.min()) < 0 or int(pairs.max()) >= self.num_blocks:  # before any collective
                raise IndexError("copy-on-write block id out of range")
            self._broadcast(OP_COW, pairs.astype(np.int32).reshape(-1))
            self.copy_on_write(out.cow)
        rec, bounds, rows, (S, T, R, W) = self.pack(out)  # every rank applies the record's table updates
        self._broadcast(OP_FORWARD, rec, bounds, greedy=1)
        self._last_n = rec.size
        self._timed_forward(bounds)
        self.steps += 1
        self._pending_rows = R
        if getattr(self, "roofline_peaks", None):
            self.roofline_s += self.step_roofline(rec, bounds, *self.roofline_peaks)
        return rows, R

    def _broadcast(self, op, rec=None, bounds=None, greedy=0):
        self.h2d_bytes += self.plane.send(op, rec, bounds, greedy)

    def greedy_picks(self, R: int):
        """Global argmax token id per logit row (device tensor [R], int32)."""
        import torch.distributed as dist

        w = self.w
        check(self.L.vllt_argmax_rows(self.logits_dev.data_ptr(), R, w.vocab_local, w.vocab_padded, w.vocab_offset,
                                      self._val.data_ptr(), self._idx.data_ptr(), _lib.stream_handle()))
        n = self.group.world
        vals, idxs = self._vals[:n * R], self._idxs[:n * R]
        dist.all_gather_into_tensor(vals, self._val[:R])
        dist.all_gather_into_tensor(idxs, self._idx[:R])
        return merge_argmax(vals.view(n, R), idxs.view(n, R))

    def gather_rows(self, rows):
        """Rank 0: full-vocabulary fp32 logits of the given logit rows of the
        last pass, [len(rows), V] on this device. Every rank takes part (the
        row list travels in one OP_GATHER message)."""
        rows = np.asarray(rows, np.int32)
        if rows.size == 0 or rows.min() < 0 or rows.max() >= self._pending_rows:
            raise IndexError("gather_rows: row outside the last pass's logit rows")
        self._broadcast(OP_GATHER, rows)
        return self._gather(int(rows.size))

    def _gather(self, n: int):
        """This rank's slice of the n rows listed at the head of the broadcast
        buffer, all-gathered into full rows."""
        import torch

        idx = self.rec_dev[:n].to(torch.int64)
        local = self.logits_dev.index_select(0, idx)[:, :self.w.vocab_local]
        return gather_vocab_rows(local, self.group.world)

    def stop_workers(self):
        self._broadcast(OP_STOP)

    def release_graphs(self):
        """Drop the captured forwards (they hold this group's NCCL calls) and
        wait for the device: must precede TPGroup.close and the process
        group's destruction, which otherwise wait on the graphs' references."""
        import gc

        import torch

        torch.cuda.synchronize(self.dev)
        self.graphs.clear()
        gc.collect()
        torch.cuda.synchronize(self.dev)

    def mark(self, tag: int):
        """Broadcast a timing mark (tag 0 = start, 1 = end); workers record a
        CUDA event, rank 0 records its own."""
        self._broadcast(OP_MARK, bounds=StepBounds(tag, 0, 0, 0, 1))
        return self._record_mark(tag)

    def _record_mark(self, tag: int):
        import torch

        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if not hasattr(self, "marks"):
            self.marks = {}
        self.marks[tag] = ev
        return ev

    def marked_seconds(self) -> float:
        self.marks[1].synchronize()
        return self.marks[0].elapsed_time(self.marks[1]) / 1e3

    # ---- ranks > 0 ------------------------------------------------------------------
    def worker_loop(self):
        """Serve rank 0's forward passes until it broadcasts the stop record.
        Runs the same dispatch as rank 0 (graph bucket or eager bounds), so
        every rank launches the same kernels and collectives."""
        import torch

        def forward(bounds, greedy):
            self._dispatch(bounds)
            if greedy:  # the merged picks at the entries rank 0's engine uses: the next
                # record may refer to them (a pass launched before rank 0 read them)
                self.picks_dev[:bounds.rows].copy_(self.greedy_picks(bounds.rows))
            torch.cuda.current_stream(self.dev).synchronize()

        def gather(n):
            self._gather(n)
            torch.cuda.current_stream(self.dev).synchronize()

        def cow(n):  # the pairs sit at the head of the broadcast buffer, on this device
            self.copy_blocks_on_device(self.rec_dev.data_ptr(), n // 2)
            torch.cuda.current_stream(self.dev).synchronize()

        return serve(self.plane, forward, self._record_mark, gather, cow)
