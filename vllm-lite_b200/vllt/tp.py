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
     global index among the maxima wins (np.argmax semantics).
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

OP_FORWARD, OP_STOP, OP_MARK = 1, 2, 3
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

        self.rec_words = self.rec_dev.numel()
        self.ctrl_host = torch.zeros(CTRL_WORDS, dtype=torch.int32, pin_memory=True)
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
        rec, bounds, rows, (S, T, R, W) = self.pack(out)
        self._reserve(S, T, R, W)
        self._broadcast(OP_FORWARD, rec, bounds, greedy=1)
        self._last_n = rec.size
        self._run(bounds)
        self.steps += 1
        self._pending_rows = R
        if getattr(self, "roofline_peaks", None):
            self.roofline_s += self.step_roofline(rec, bounds, *self.roofline_peaks)
        return rows, R

    def _broadcast(self, op, rec=None, bounds=None, greedy=0):
        import torch.distributed as dist

        n = 0 if rec is None else rec.size
        if rec is not None:
            self.rec_host[:n].numpy()[:] = rec
        b = bounds or StepBounds(0, 0, 0, 0, 1)
        self.rec_host[-CTRL_WORDS:].numpy()[:] = [op, b.tokens, b.rows, b.decode_seqs, b.tiles, b.max_ctx, greedy, n]
        if n:
            self.rec_dev[:n].copy_(self.rec_host[:n], non_blocking=True)
        self.rec_dev[-CTRL_WORDS:].copy_(self.rec_host[-CTRL_WORDS:], non_blocking=True)
        self.h2d_bytes += 4 * (n + CTRL_WORDS)
        dist.broadcast(self.rec_dev, src=0)

    def _run(self, bounds):
        if self.use_graphs:
            self._forward_graph(bounds)
        else:
            self._forward(bounds)

    def greedy_picks(self, R: int):
        """Global argmax token id per logit row (device tensor [R], int32)."""
        import torch
        import torch.distributed as dist

        w = self.w
        check(self.L.vllt_argmax_rows(self.logits_dev.data_ptr(), R, w.vocab_local, w.vocab_padded, w.vocab_offset,
                                      self._val.data_ptr(), self._idx.data_ptr(), _lib.stream_handle()))
        n = self.group.world
        vals, idxs = self._vals[:n * R], self._idxs[:n * R]
        dist.all_gather_into_tensor(vals, self._val[:R])
        dist.all_gather_into_tensor(idxs, self._idx[:R])
        vals, idxs = vals.view(n, R), idxs.view(n, R)
        best = vals.max(0).values
        # ties: the lowest rank holds the lowest global index (first max wins)
        score = torch.where(vals == best, torch.arange(n, 0, -1, device=self.dev).view(n, 1), 0)
        return idxs.gather(0, score.argmax(0, keepdim=True)).view(R)

    def stop_workers(self):
        self._broadcast(OP_STOP)

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
        """Serve rank 0's forward passes until it broadcasts the stop record."""
        import torch
        import torch.distributed as dist

        while True:
            dist.broadcast(self.rec_dev, src=0)
            self.ctrl_host.copy_(self.rec_dev[-CTRL_WORDS:])
            ctrl = self.ctrl_host.numpy()
            if ctrl[0] == OP_STOP:
                break
            if ctrl[0] == OP_MARK:
                self._record_mark(int(ctrl[1]))
                continue
            bounds = StepBounds(*[int(x) for x in ctrl[1:6]])
            self._run(bounds)
            if ctrl[6]:
                self.greedy_picks(int(ctrl[2]))
            torch.cuda.current_stream(self.dev).synchronize()
